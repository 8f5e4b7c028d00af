// act_quant's arithmetic on 1x128 blocks of a bf16 row, shared by the FP8 layer
// (fp8_moe.cu), the V4 layer and the dense FP8 linear (fp8_linear.cu).
//
// Reference: act_quant, vendor/deepseek_v4_ref/inference/kernel.py:40-125 and its
// CPU restatement engines/deepseek_v4/v4_kernels_cpu.py:68-104 -- per block the
// amax floored at 1e-4, the scale amax/448 in fp32 (checkpoints without
// scale_fmt) or 2^ceil(log2(amax/448)) (scale_fmt "ue8m0"), the elements x/scale
// saturated to e4m3.
#pragma once
#include <cuda_fp8.h>

#include "common.cuh"

namespace flyai {

// fp32 1/448 as torch forms it for `amax * (1.0 / FP8_MAX)` on an fp32 tensor.
constexpr float kF8Inv448 = static_cast<float>(1.0 / 448.0);

__device__ __forceinline__ uint32_t f32_to_e4m3(float v) {
  v = fminf(fmaxf(v, -448.f), 448.f);
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// The ue8m0 activation scale of a 128-block with maximum |x| = amax:
// 2^ceil(log2(max(amax, 1e-4) * (1/448))), exact at powers of two (the
// reference's fast_round_scale, engines/deepseek_v4/v4_kernels_cpu.py:68-76).
// Returns the exponent; the scale is 2^exponent.
__device__ __forceinline__ int ue8m0_exp(float amax, float inv448) {
  const uint32_t b = __float_as_uint(__fmul_rn(fmaxf(amax, 1e-4f), inv448));
  const int e = static_cast<int>((b >> 23) & 0xFFu) - 127;
  return e + ((b & 0x7FFFFFu) != 0u ? 1 : 0);
}
__device__ __forceinline__ float exp2_int(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

// One warp quantises the 128-element block at src (bf16, 8-byte aligned): lane l
// gets the e4m3 bytes of elements 4l..4l+3 (element 4l in the low byte), every
// lane the block's scale.
__device__ __forceinline__ uint32_t act_quant4(const uint16_t* src, int lane, int ue8m0, float& s) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(src + lane * 4));
  const float v[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u),
                      __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xFFFF0000u)};
  float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  a = fmaxf(warp_max(a), 1e-4f);
  s = ue8m0 ? exp2_int(ue8m0_exp(a, kF8Inv448)) : __fmul_rn(a, kF8Inv448);
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) packed |= f32_to_e4m3(__fdiv_rn(v[j], s)) << (8 * j);
  return packed;
}

}  // namespace flyai
