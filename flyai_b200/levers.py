"""One registry of this package's levers, comparing "requested" with "observed".

Each drop-in lever (the GPT-OSS mlp, the DeepSeek MoE.forward, the M2.5 stage
moe, the K3 moe_infer) is switched by an environment flag its module parses at import.  Two facts
are kept per lever and compared, as the reference's lever registry does
(engines/deepseek_v4/v4_levers.py:1-40):

* requested -- the flag as the owning module parsed it (what the process obeys,
  not os.environ: a flag set after import does not count), for a lever whose
  install was called;
* observed  -- what is live: a forward rebound by the lever, a stage module
  replaced.

``audit()`` returns one row per lever with a verdict: OK, UNUSED (no install call
and no flag set), MISMATCH (requested and observed disagree; the environment says
something the module did not parse; or the flag is set on and nothing was
installed) or UNKNOWN (a FLYAI_MOE_* variable nothing here reads).  ``report()``
prints the rows; with FLYAI_MOE_LEVERS_STRICT=1 ``check()`` raises on any
finding.
"""
import os

from . import deepseek, gpt_oss, k3, m25

# flags read by the shared library or the tools rather than by a lever
_OTHER_FLAGS = {"FLYAI_MOE_CHECK", "FLYAI_MOE_LEVERS_STRICT"}


def _levers():
    # env flag -> (name, module flag, install calls, installed now)
    return {
        "FLYAI_MOE_B200": ("gpt-oss mlp (GptOssMLP.forward)", lambda: gpt_oss.ENABLED,
                           gpt_oss.attempts, lambda: gpt_oss.installed_count() > 0),
        "FLYAI_MOE_DEEPSEEK": ("deepseek MoE.forward", lambda: deepseek.ENABLED,
                               deepseek.attempts, lambda: len(deepseek.installed()) > 0),
        "FLYAI_MOE_M25": ("minimax-m2.5 stage moe", lambda: m25.ENABLED,
                          m25.attempts, lambda: len(m25.installed()) > 0),
        "FLYAI_MOE_K3": ("kimi-k3 moe_infer", lambda: k3.ENABLED,
                         k3.attempts, lambda: len(k3.installed()) > 0),
    }


def _env_on(v):
    return v not in ("", "0")


def audit(environ=None):
    environ = os.environ if environ is None else environ
    rows = []
    levers = _levers()
    for env, (name, flag, attempts, observed) in levers.items():
        req, obs = bool(flag()) and attempts() > 0, bool(observed())
        verdict = "OK"
        if env in environ and _env_on(environ[env]) != bool(flag()):
            verdict = "MISMATCH"   # the flag changed after the module parsed it
        elif attempts() == 0 and not obs:
            verdict = "MISMATCH" if env in environ and _env_on(environ[env]) else "UNUSED"
        elif req != obs:
            verdict = "MISMATCH"
        rows.append({"lever": name, "env": env, "env_value": environ.get(env),
                     "requested": req, "observed": obs, "verdict": verdict})
    for k in sorted(environ):
        if k.startswith("FLYAI_MOE_") and k not in levers and k not in _OTHER_FLAGS:
            rows.append({"lever": None, "env": k, "env_value": environ[k], "requested": None,
                         "observed": None, "verdict": "UNKNOWN"})
    return rows


def report(environ=None):
    return "\n".join(f"{r['verdict']:8s} {r['env']}={r['env_value']!s:5s} "
                     f"requested={r['requested']} observed={r['observed']}  {r['lever'] or ''}"
                     for r in audit(environ))


def check(environ=None):
    """Raise when any lever's requested and observed state disagree (or an unknown
    flag is set) and FLYAI_MOE_LEVERS_STRICT=1; returns the audit rows."""
    environ = os.environ if environ is None else environ
    rows = audit(environ)
    bad = [r for r in rows if r["verdict"] not in ("OK", "UNUSED")]
    if bad and _env_on(environ.get("FLYAI_MOE_LEVERS_STRICT", "0")):
        raise RuntimeError("lever findings:\n" + report(environ))
    return rows
