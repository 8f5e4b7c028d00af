// Shared pieces of the tcgen05 expert kernels (tc_experts.cu: verify sizes,
// tc_prefill.cu: prefill sizes): the packed bank layout, a projection's
// operands and the walk over a CTA's (chunk, tile) work items.
#pragma once
#include "common.cuh"
#include "terms.cuh"

namespace flyai {

// ---------------------------------------------------------------------------
// Packed bank
// ---------------------------------------------------------------------------
// Per expert, rows are cut into M-tiles of 128 (the MMA's M) and K into K-tiles
// of kKT elements.  Tile (mt, kt) holds its e2m1 data in canonical K-major
// layout -- 16-byte chunk c (one 32-element scale group) of row r at
// c * rows_t * 16 + (r / 8) * 128 + (r % 8) * 16 -- followed by its e8m0 scales
// in 512-byte chunks of 128 rows x 4 groups (row r, group g at
// (r % 32) * 16 + (r / 32) * 4 + g % 4), the layout tcgen05.cp copies into TMEM.
// Rows of the last M-tile past the expert's end are absent from the bank; the
// MMA computes garbage for those lanes and the epilogue ignores them.
constexpr int kKT = 512;

struct TcLayout {
  int R, K, G, MT, NKT, last_rows;
  size_t tile_full, mtile_full, mtile_last, expert_bytes;
};

__host__ __device__ inline size_t tc_tile_bytes(int rows, int kt_len) {
  return static_cast<size_t>(rows) * (kt_len / 2) + static_cast<size_t>((kt_len + 127) / 128) * 512;
}
__host__ __device__ inline int tc_kt_len(const TcLayout& L, int kt) {
  return L.K - kt * kKT < kKT ? L.K - kt * kKT : kKT;
}
__host__ __device__ inline int tc_rows(const TcLayout& L, int mt) {
  return mt == L.MT - 1 ? L.last_rows : 128;
}
__host__ __device__ inline size_t tc_mtile_bytes(const TcLayout& L, int rows) {
  size_t b = 0;
  for (int kt = 0; kt < L.NKT; ++kt) b += tc_tile_bytes(rows, tc_kt_len(L, kt));
  return b;
}
__host__ __device__ inline size_t tc_tile_offset(const TcLayout& L, int mt, int kt) {
  return static_cast<size_t>(mt) * L.mtile_full +
         static_cast<size_t>(kt) * tc_tile_bytes(tc_rows(L, mt), kKT);
}

inline TcLayout tc_layout(const flyai_moe_desc& d, int proj) {
  TcLayout L{};
  L.R = proj == FLYAI_PROJ_W13 ? 2 * d.inter : d.hidden;
  L.K = proj == FLYAI_PROJ_W13 ? d.hidden : d.inter;
  L.G = L.K / 32;
  L.MT = (L.R + 127) / 128;
  L.last_rows = L.R - 128 * (L.MT - 1);
  L.NKT = (L.K + kKT - 1) / kKT;
  L.tile_full = tc_tile_bytes(128, kKT);
  L.mtile_full = tc_mtile_bytes(L, 128);
  L.mtile_last = tc_mtile_bytes(L, L.last_rows);
  L.expert_bytes = static_cast<size_t>(L.MT - 1) * L.mtile_full + L.mtile_last;
  return L;
}

// Tensor-memory columns of the verify kernel: 4 accumulators x 2 halves x 32,
// 16 per ring stage for A scales, then two buffers of 4 per 128-element K group
// for B scales -- 512 in all, so K <= 3072 (the prefill kernel fits inside).
constexpr int kTcMaxK = 3072;
constexpr int kTcBlockBytes = kTerms * 16;                 // one 32-element block of a term row

struct TcProj {
  const uint8_t* bank;
  TcLayout L;
  const float* bias;          // [El, R] or null
  const uint8_t* act_terms;   // activation rows of term_row_bytes(K)
  const uint8_t* act_sf;      // activation rows of term_sf_row_bytes(K)
};

struct TcItem {
  int gu, chunk, mt;
};
__device__ __forceinline__ bool tc_same_b(const TcItem& a, const TcItem& b) {
  return a.gu == b.gu && a.chunk == b.chunk;
}
// Walks this CTA's items: gate/up [g0, g0 + ng) then down [d0, d0 + nd), with
// no divisions after the start (single-thread issue loops are latency bound).
struct TcCursor {
  TcItem t;
  long long left_gu, left_dn;
  int mtg, mtd;
  long long d0;
  __device__ __forceinline__ void start(long long g0, long long ng, long long d0_, long long nd,
                                        int mtg_, int mtd_) {
    mtg = mtg_;
    mtd = mtd_;
    d0 = d0_;
    left_gu = ng;
    left_dn = nd;
    if (ng > 0) {
      t = TcItem{1, static_cast<int>(g0 / mtg), static_cast<int>(g0 % mtg)};
    } else {
      t = TcItem{0, static_cast<int>(d0 / mtd), static_cast<int>(d0 % mtd)};
    }
  }
  __device__ __forceinline__ bool valid() const { return left_gu + left_dn > 0; }
  __device__ __forceinline__ void next() {
    if (t.gu) {
      if (--left_gu == 0) {
        t = TcItem{0, static_cast<int>(d0 / mtd), static_cast<int>(d0 % mtd)};
        return;
      }
      if (++t.mt == mtg) {
        t.mt = 0;
        ++t.chunk;
      }
    } else {
      --left_dn;
      if (++t.mt == mtd) {
        t.mt = 0;
        ++t.chunk;
      }
    }
  }
  // does the item after the current one use the same B (same phase and chunk)?
  __device__ __forceinline__ bool next_same_b() const {
    if (t.gu) return left_gu > 1 && t.mt + 1 < mtg;
    return left_dn > 1 && t.mt + 1 < mtd;
  }
};

// Prefill order: CTA b takes gate/up items b, b+G, b+2G, ... (item = chunk * NI +
// row block), then down items the same way.  At any time consecutive CTAs work on
// the row blocks of the same few chunks, so a chunk's activation rows, and the
// weights of an expert whose chunks are adjacent, are fetched once into L2 and
// shared; every CTA still finishes its gate/up items before its first down item.
struct TcStridedCursor {
  TcItem t;
  long long u, n_gu, n_dn;   // current item number within its phase; items per phase
  int b, G, NI, NT;
  __device__ __forceinline__ void start(int b_, int G_, long long nch, int NI_, int NT_) {
    b = b_, G = G_, NI = NI_, NT = NT_;
    n_gu = nch * NI, n_dn = nch * NT;
    u = b;
    t.gu = 1;
    if (u >= n_gu) {
      t.gu = 0;
      u = b;
    }
    set();
  }
  __device__ __forceinline__ void set() {
    const int n = t.gu ? NI : NT;
    t.chunk = static_cast<int>(u / n);
    t.mt = static_cast<int>(u - static_cast<long long>(t.chunk) * n);
  }
  __device__ __forceinline__ bool valid() const { return u < (t.gu ? n_gu : n_dn); }
  __device__ __forceinline__ void next() {
    u += G;
    if (t.gu && u >= n_gu) {   // gate/up done: first down item of this CTA
      t.gu = 0;
      u = b;
    }
    if (valid()) set();
  }
  // does the item after the current one use the same B (same phase and chunk)?
  __device__ __forceinline__ bool next_same_b() const {
    const long long v = u + G;
    if (v >= (t.gu ? n_gu : n_dn)) return false;
    return v / (t.gu ? NI : NT) == t.chunk;
  }
};

// Verify order: runs of `run` consecutive items (in chunk-major order) dealt
// round-robin -- CTA b takes runs b, b+G, ... of the gate/up items, then of
// the down items.  A round covers a few whole chunks, so a chunk's gate/up tiles
// finish together early in the phase and its down tiles, dealt later, find them
// done; within a run the chunk (and its B operand) mostly stays the same.  With
// few items per CTA a run of 1 spreads them over more SMs.
struct TcRunCursor {
  TcItem t;
  long long u, n_gu, n_dn;   // item number within its phase; items per phase
  int b, G, NI, NT, run;
  __device__ __forceinline__ void start(int b_, int G_, long long nch, int NI_, int NT_, int run_) {
    b = b_, G = G_, NI = NI_, NT = NT_, run = run_;
    n_gu = nch * NI, n_dn = nch * NT;
    t.gu = 1;
    u = static_cast<long long>(b) * run;
    if (u >= n_gu) t.gu = 0;   // no gate/up run for this CTA: its first down run
    set();
  }
  __device__ __forceinline__ void set() {
    const int n = t.gu ? NI : NT;
    t.chunk = static_cast<int>(u / n);
    t.mt = static_cast<int>(u - static_cast<long long>(t.chunk) * n);
  }
  __device__ __forceinline__ long long n_phase() const { return t.gu ? n_gu : n_dn; }
  __device__ __forceinline__ bool valid() const { return u < n_phase(); }
  // the item after v in this CTA's walk of the current phase: the next one of
  // the run, else the first of the CTA's next run
  __device__ __forceinline__ long long after(long long v) const {
    return ((v + 1) % run != 0 && v + 1 < n_phase()) ? v + 1
                                                     : v - v % run + static_cast<long long>(G) * run;
  }
  __device__ __forceinline__ void next() {
    u = after(u);
    if (t.gu && u >= n_gu) {   // gate/up done: first down run of this CTA
      t.gu = 0;
      u = static_cast<long long>(b) * run;
    }
    if (valid()) set();
  }
  // does the item after the current one use the same B (same phase and chunk)?
  __device__ __forceinline__ bool next_same_b() const {
    const long long v = after(u);
    if (v >= n_phase()) return false;
    return v / (t.gu ? NI : NT) == t.chunk;
  }
};

}  // namespace flyai
