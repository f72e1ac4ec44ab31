"""CPU ORACLE for the tokengate_b200 gated-prefill path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this package, and only as the checker or the timed CPU
baseline; the product (tokengate_b200) never imports it and has no CPU path.

Contents (each function cites the reference code it restates):
  * attention.py  — causal GQA attention with an additive per-key bias, float64
                    numpy (reference: sdpa_compat.sdpa_causal and the flex
                    score_mod);
  * tg_oracle.c   — the fixed-order fp32 gate scorer and the top-K /
                    keep-list / bias-row construction (bit-exact contracts);
  * select.py     — ctypes bindings of tg_oracle.c plus numpy versions of the
                    selection and the row compaction;
  * prefill.py    — the gated prefill (Phase 1 -> score -> select -> compact
                    -> Phase 2 -> first token) on CPU in float32 torch.

Parity of the oracle with the reference itself is pinned by
tests/test_oracle.py against fixtures under tests/golden/ that
tests/golden/make_golden.py produced by running the reference's own Python
code (sdpa_compat, FlexAttention score_mod, _select_indices, keep-list,
build_gate_bias_vectorized, prefill_batch_for_decode) in this container.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "liboracle.so")
SRC = os.path.join(HERE, "tg_oracle.c")


def build(force: bool = False) -> str:
    """Compile tg_oracle.c with gcc (no FP contraction) into oracle/_build/."""
    if not force and os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= os.path.getmtime(SRC):
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = ["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           SRC, "-o", tmp, "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH
