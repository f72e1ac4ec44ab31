"""CPU ORACLE (test infrastructure): the finalized TokenGate gate (E2EGate).

Restates, in numpy float32 with the reference's bf16 rounding points:
  * branch_score   — the scoring branch's readout over a fused [gate | up] row,
                     bf16(sum_k bf16(bf16(silu(g_k)) * u_k) * w_k) (gate_branch_hs,
                     tokengate/e2e_gate/gate_module/gate_forward.py:491-524 with the
                     absorbed 1-row down_proj :330-340), by ctypes into tg_oracle.c
                     (the kernel's summation order, bit-exact contract);
  * e2e_bias       — E2EGate.forward: sequence RMSNorm of the raw scores (Qwen3RMSNorm(1),
                     eps 1e-6, gain) times softplus(gate_scale) -> (n, L', H)
                     (e2e_gate_module.py:327-385);
  * aggregate      — slot 0, mean over heads (e2e_gate_module.py:387-399);
  * select         — torch.topk of the aggregate (gate_forward.py:84-99, :127-143)
                     ordered (value desc, index asc);
  * ssmax_ratio    — r = clamp(log m / log(p + 1), <= 1) (gate_forward.py:574-585);
  * phase2_tables  — per layer l and head h: s_eff = bf16(bf16(S_eff[l,h]) * bf16(r)),
                     bias = bf16(bf16(b) * bf16(mean_h s_eff)) with b = 0 off the state
                     span and bf16(-1e9) in pads (build_gate_bias_vectorized
                     :968-1000, pads :1463-1469, _apply_gate_bias :588-660,
                     _ssmax_s_eff / _phase2_q_bias qwen3_flex_attention.py:417-473).
Pinned against tests/golden/e2e_gate.npz (the reference's own E2EGate,
_ssmax_ratio and _phase2_q_bias outputs).
"""
import ctypes

import numpy as np

from . import select as _sel

_RMS_EPS = 1e-6


def _c():
    lib = _sel._c()
    if not getattr(lib, "_e2e_ready", False):
        lib.oracle_branch_score.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_void_p]
        lib.oracle_branch_score.restype = None
        lib.oracle_silu.argtypes = [ctypes.c_float]
        lib.oracle_silu.restype = ctypes.c_float
        lib._e2e_ready = True
    return lib


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32 (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def branch_score(gu_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """gu_bits: (n, >= 2*inter) uint16 bf16 patterns [g | u]; w_bits: (inter,) -> (n,) fp32."""
    gu = np.ascontiguousarray(gu_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    n, ld = gu.shape
    inter = w.shape[0]
    if inter % 256 or ld < 2 * inter:
        raise ValueError("inter must be a multiple of 256 and rows hold [g | u]")
    out = np.empty(n, dtype=np.float32)
    _c().oracle_branch_score(gu.ctypes.data, ld, n, inter, w.ctypes.data, out.ctypes.data)
    return out


def silu(g: np.ndarray) -> np.ndarray:
    f = _c().oracle_silu
    g = np.asarray(g, dtype=np.float32)
    return np.array([f(float(x)) for x in g.ravel()], dtype=np.float32).reshape(g.shape)


def softplus(x: np.ndarray) -> np.ndarray:
    """torch's softplus (beta 1, threshold 20) in float64, rounded to float32."""
    x = np.asarray(x, dtype=np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def seq_rms_scale(raw: np.ndarray, eps: float = _RMS_EPS) -> np.float32:
    """rsqrt(mean(x^2) + eps) of one request's raw scores (float64, rounded to float32)."""
    x = np.asarray(raw, dtype=np.float64)
    return np.float32(1.0 / np.sqrt(np.mean(x * x) + eps))


def e2e_bias(raw: np.ndarray, gate_scale_eff: np.ndarray, eps: float = _RMS_EPS,
             gain: float = 1.0) -> np.ndarray:
    """(n,) raw scores -> (n, L', H) fp32 bias of E2EGate.forward."""
    x = np.asarray(raw, dtype=np.float32)
    bn = np.float32(gain) * (x * seq_rms_scale(x, eps))
    return (bn[:, None, None] * np.asarray(gate_scale_eff, dtype=np.float32)[None]).astype(np.float32)


def aggregate(b: np.ndarray) -> np.ndarray:
    """(n, L', H) -> (n,): slot 0, uniform mean over heads (sum of b * (1/H))."""
    b0 = b[:, 0, :]
    H = b0.shape[1]
    if H == 1:
        return b0[:, 0]
    w = np.float32(1.0 / H)
    acc = np.zeros(b0.shape[0], dtype=np.float32)
    for h in range(H):
        acc = (acc + b0[:, h] * w).astype(np.float32)
    return acc


def select(agg: np.ndarray, k: int) -> np.ndarray:
    """Top-k indices of the aggregate, ascending; rank (value desc, index asc), -0 == +0."""
    return _sel.topk_indices(np.asarray(agg, dtype=np.float32) + np.float32(0.0), k)


def ssmax_ratio(kept_positions: np.ndarray) -> np.ndarray:
    """(B, n) int64 kept positions (pads included) -> r (B, n) fp32."""
    kp = np.asarray(kept_positions)
    n = kp.shape[-1]
    m = np.maximum(np.arange(1, n + 1, dtype=np.float32), np.float32(2.0))
    p = np.maximum(kp.astype(np.float32) + np.float32(1.0), np.float32(2.0))
    r = (np.log(m)[None, :] / np.log(p)).astype(np.float32)
    return np.minimum(r, np.float32(1.0))


def phase2_tables(raws, starts, n_kept, kept_positions, gate_scale_eff, attn_scale_eff,
                  eps: float = _RMS_EPS, gain: float = 1.0):
    """Per-layer Phase-2 bias and query scale, each (L', B, H, n_alloc) fp32.

    raws: per request, the raw scores of its state span; starts: state begins;
    n_kept: kept counts; kept_positions: (B, n_alloc) int64 (pads 0)."""
    kp = np.asarray(kept_positions)
    B, n_alloc = kp.shape
    gs = np.asarray(gate_scale_eff, dtype=np.float32)
    S = bf16_round(np.asarray(attn_scale_eff, dtype=np.float32))
    L, H = gs.shape
    r = bf16_round(ssmax_ratio(kp))                                         # (B, n)
    s_eff = bf16_round(S[:, None, :, None] * r[None, :, None, :])           # (L, B, H, n)
    acc = np.zeros((L, B, n_alloc), dtype=np.float32)
    for h in range(H):
        acc = (acc + s_eff[:, :, h, :]).astype(np.float32)
    sb = bf16_round(acc * np.float32(1.0 / H))                              # (L, B, n)
    base = np.zeros((L, B, H, n_alloc), dtype=np.float32)
    for b in range(B):
        raw = np.asarray(raws[b], dtype=np.float32)
        bias_b = bf16_round(e2e_bias(raw, gs, eps, gain))                   # (n_state, L, H)
        n = n_kept[b]
        pos = kp[b, :n]
        st = (pos >= starts[b]) & (pos < starts[b] + len(raw))
        cols = np.nonzero(st)[0]
        vals = bias_b[pos[cols] - starts[b]]                                # (nc, L, H)
        for l in range(L):
            base[l, b][:, cols] = vals[:, l, :].T
        base[:, b, :, n:] = bf16_round(np.float32(-1e9))
    bias = bf16_round(base * sb[:, :, None, :])
    return bias, s_eff
