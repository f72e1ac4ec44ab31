"""CPU ORACLE (test infrastructure): gate scoring, top-K selection, compaction.

  gate_score      — ctypes call of tg_oracle.c's fixed-order fp32 scorer
                    (restates b_scores = logsigmoid(readout(h_art.to(fp32))),
                     tokengate/e2e_gate/gate_module/gate_forward.py:1396-1407);
  topk_select     — the selection + keep-list + bias row of one request:
                    torch.topk(score, K_clamped) (gate_forward.py:84-99),
                    keep = [0,start) ++ start+sort(topk) ++ [end,len) (:1417-1421),
                    gate_bias = score at kept state tokens, 0 elsewhere, -1e9 pads
                    (:968-1036, :1463-1469); order (score desc, index asc).
                    Two independent versions: numpy (stable lexsort) and C.
  gather_rows     — hs_pruned[b, :n] = hs[b, keep] with zero rows past n
                    (:1443-1461) and the K/V index_select + pad (:1491-1522).
"""
import ctypes

import numpy as np

from . import LIB_PATH, build

_lib = None


def _c():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.oracle_gate_score.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        _lib.oracle_gate_score.restype = None
        _lib.oracle_topk_select.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib.oracle_topk_select.restype = ctypes.c_int64
        _lib.oracle_logsigmoid.argtypes = [ctypes.c_float]
        _lib.oracle_logsigmoid.restype = ctypes.c_float
    return _lib


def logsigmoid(z: np.ndarray) -> np.ndarray:
    """Elementwise fp32 logsigmoid with the kernel's IEEE-only evaluation."""
    f = _c().oracle_logsigmoid
    z = np.asarray(z, dtype=np.float32)
    return np.array([f(float(x)) for x in z.ravel()], dtype=np.float32).reshape(z.shape)


def gate_score(h_bf16_bits: np.ndarray, w: np.ndarray) -> np.ndarray:
    """h_bf16_bits: (n, H) uint16 (bf16 bit patterns); w: (H,) fp32 -> (n,) fp32."""
    h = np.ascontiguousarray(h_bf16_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, H = h.shape
    if H % 256:
        raise ValueError("hidden size must be a multiple of 256")
    out = np.empty(n, dtype=np.float32)
    _c().oracle_gate_score(h.ctypes.data, H, n, H, w.ctypes.data, out.ctypes.data)
    return out


def order_keys(scores: np.ndarray) -> np.ndarray:
    """IEEE total order of fp32 values as uint32 (-0.0 < +0.0)."""
    u = np.asarray(scores, dtype=np.float32).view(np.uint32)
    return np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def topk_indices(scores: np.ndarray, k: int) -> np.ndarray:
    """The k state-relative indices kept, ascending; rank by (score desc, index asc)."""
    keys = order_keys(scores).astype(np.int64)
    idx = np.arange(len(keys))
    order = np.lexsort((idx, -keys))
    return np.sort(order[:k])


def topk_select(scores: np.ndarray, k: int, state_begin: int, seq_len: int, n_alloc: int,
                use_c: bool = False):
    """(keep int64 (n_alloc,), bias fp32 (n_alloc,), topk_local int64 (k,), n_kept)."""
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    n = len(scores)
    if use_c:
        keep = np.empty(n_alloc, dtype=np.int64)
        bias = np.empty(n_alloc, dtype=np.float32)
        tl = np.empty(k, dtype=np.int64)
        nk = _c().oracle_topk_select(scores.ctypes.data, n, k, state_begin, seq_len, n_alloc,
                                     keep.ctypes.data, bias.ctypes.data, tl.ctypes.data)
        if nk < 0:
            raise ValueError("bad selection arguments")
        return keep, bias, tl, int(nk)
    tl = topk_indices(scores, k)
    state_end = state_begin + n
    kept = np.concatenate([np.arange(state_begin), state_begin + tl, np.arange(state_end, seq_len)])
    nk = len(kept)
    if nk > n_alloc:
        raise ValueError("n_kept exceeds n_alloc")
    keep = np.zeros(n_alloc, dtype=np.int64)
    keep[:nk] = kept
    bias = np.full(n_alloc, -1e9, dtype=np.float32)
    bias[:nk] = 0.0
    bias[state_begin:state_begin + k] = scores[tl]
    return keep, bias, tl.astype(np.int64), nk


def gather_rows(src: np.ndarray, idx: np.ndarray, n_valid: int, n_rows: int, axis: int = 0) -> np.ndarray:
    """dst[r] = src[idx[r]] along `axis` for r < n_valid, zeros for n_valid <= r < n_rows."""
    src = np.asarray(src)
    shape = list(src.shape)
    shape[axis] = n_rows
    dst = np.zeros(shape, dtype=src.dtype)
    sl = [slice(None)] * src.ndim
    sl[axis] = slice(0, n_valid)
    dst[tuple(sl)] = np.take(src, np.asarray(idx[:n_valid]), axis=axis)
    return dst
