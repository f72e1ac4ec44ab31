"""Torch-facing wrappers of the four hot-path kernels.

Each wrapper validates tensors, takes raw pointers and strides, and calls the
C ABI on the current CUDA stream of the tensors' device. All outputs are
allocated here by torch (the C ABI allocates nothing). No wrapper has a CPU
or eager fallback: CPU tensors, a missing library or an unsupported shape
raise.
"""
from typing import Optional, Sequence, Tuple

import contextlib
import ctypes

import torch

from . import _lib

_LOG2E = 1.4426950408889634


def _require_cuda(name: str, t: torch.Tensor, dtype: Optional[torch.dtype] = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the B200 kernels have no CPU path), "
                         f"got {t.device}")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


def _device_ctx(t: torch.Tensor):
    if torch.cuda.current_device() == t.device.index:
        return contextlib.nullcontext()
    return torch.cuda.device(t.device)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _i32_array(values: Sequence[int]):
    arr = (ctypes.c_int32 * len(values))(*[int(v) for v in values])
    return arr


# ----------------------------------------------------------------- attention
def keybias_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      bias: Optional[torch.Tensor] = None,
                      softmax_scale: Optional[float] = None,
                      causal: bool = True,
                      q_row_scale: Optional[torch.Tensor] = None,
                      return_lse: bool = False,
                      out: Optional[torch.Tensor] = None):
    """softmax(scale * q k^T + bias) v with causal masking and GQA.

    q: (B, Sq, Hq, 128) bf16, k/v: (B, Sk, Hkv, 128) bf16, any strides with a
    contiguous last dim (the (B, H, S, D) views the reference passes are the
    transposes of these). bias: fp32, broadcastable to (B, Hq, Sk) with a
    contiguous last dim, in score units (what the FlexAttention score_mod
    adds). q_row_scale: fp32 broadcastable to (B, Hq, Sq) with a contiguous
    last dim. Returns out (B, Sq, Hq, 128) bf16, and lse (B, Hq, Sq) fp32 when
    return_lse.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t, torch.bfloat16)
        if t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be 4-D (B, S, H, D) with a contiguous last dim")
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    if k.shape[0] != B or v.shape[:3] != k.shape[:3] or k.shape[3] != D or v.shape[3] != D:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)}")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on one device")
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if out is None:
        out = torch.empty((B, Sq, Hq, D), dtype=torch.bfloat16, device=q.device)
    else:
        _require_cuda("out", out, torch.bfloat16)
        if tuple(out.shape) != (B, Sq, Hq, D) or out.stride(-1) != 1:
            raise ValueError("out must be (B, Sq, Hq, D) with a contiguous last dim")
    lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=q.device) if return_lse else None

    bias_ptr, bsb, bsh = None, 0, 0
    if bias is not None:
        _require_cuda("bias", bias, torch.float32)
        bb = bias
        while bb.dim() < 3:
            bb = bb.unsqueeze(0)
        if bb.dim() != 3 or bb.shape[-1] != Sk or bb.stride(-1) != 1:
            raise ValueError(f"bias must broadcast to (B, Hq, Sk)=({B}, {Hq}, {Sk}) with a "
                             f"contiguous last dim, got {tuple(bias.shape)}")
        if bb.shape[0] not in (1, B) or bb.shape[1] not in (1, Hq):
            raise ValueError(f"bias shape {tuple(bias.shape)} does not broadcast to ({B}, {Hq}, {Sk})")
        bsb = 0 if bb.shape[0] == 1 else bb.stride(0)
        bsh = 0 if bb.shape[1] == 1 else bb.stride(1)
        bias_ptr = bb.data_ptr()
    qs_ptr, qsb, qsh = None, 0, 0
    if q_row_scale is not None:
        _require_cuda("q_row_scale", q_row_scale, torch.float32)
        qq = q_row_scale
        while qq.dim() < 3:
            qq = qq.unsqueeze(0)
        if qq.shape[-1] != Sq or qq.stride(-1) != 1 or qq.shape[0] not in (1, B) \
                or qq.shape[1] not in (1, Hq):
            raise ValueError(f"q_row_scale must broadcast to ({B}, {Hq}, {Sq}) with a contiguous last dim")
        qsb = 0 if qq.shape[0] == 1 else qq.stride(0)
        qsh = 0 if qq.shape[1] == 1 else qq.stride(1)
        qs_ptr = qq.data_ptr()

    L = _lib.lib()
    with _device_ctx(q):
        _lib.check_launch(L.tg_keybias_attn_fwd(
            q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
            v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
            bias_ptr, bsb, bsh,
            qs_ptr, qsb, qsh,
            out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
            lse.data_ptr() if lse is not None else None,
            lse.stride(0) if lse is not None else 0, lse.stride(1) if lse is not None else 0,
            B, Sq, Sk, Hq, Hkv, D, float(softmax_scale), int(bool(causal)), _stream(q)))
    return (out, lse) if return_lse else out


# ----------------------------------------------------------------- gate score
def gate_score(hidden: torch.Tensor, w: torch.Tensor, row_begin: Sequence[int],
               row_count: Sequence[int], out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """scores[b, r] = logsigmoid(w . hidden[b, row_begin[b] + r]) for r < row_count[b].

    hidden: (B, S, H) bf16 with a contiguous last dim; w: (H,) fp32 contiguous.
    Returns fp32 (B, max(row_count)); entries past row_count[b] are untouched
    (zero when the output is allocated here).
    """
    _require_cuda("hidden", hidden, torch.bfloat16)
    _require_cuda("w", w, torch.float32)
    if hidden.dim() != 3 or hidden.stride(-1) != 1:
        raise ValueError("hidden must be (B, S, H) with a contiguous last dim")
    B, S, H = hidden.shape
    if w.dim() != 1 or w.shape[0] != H or not w.is_contiguous():
        raise ValueError(f"w must be a contiguous ({H},) vector")
    if len(row_begin) != B or len(row_count) != B:
        raise ValueError("row_begin / row_count need one entry per request")
    for b in range(B):
        if row_begin[b] < 0 or row_count[b] < 0 or row_begin[b] + row_count[b] > S:
            raise ValueError(f"request {b}: rows [{row_begin[b]}, {row_begin[b] + row_count[b]}) "
                             f"outside [0, {S})")
    n_max = max(int(c) for c in row_count)
    if out is None:
        out = torch.zeros((B, max(n_max, 1)), dtype=torch.float32, device=hidden.device)
    else:
        _require_cuda("out", out, torch.float32)
        if out.dim() != 2 or out.shape[0] != B or out.shape[1] < n_max or out.stride(1) != 1:
            raise ValueError("out must be (B, >= max(row_count)) fp32 with a contiguous last dim")
    L = _lib.lib()
    with _device_ctx(hidden):
        _lib.check_launch(L.tg_gate_score(hidden.data_ptr(), hidden.stride(0), hidden.stride(1), H,
                                   w.data_ptr(), B, _i32_array(row_begin), _i32_array(row_count),
                                   out.data_ptr(), out.stride(0), _stream(hidden)))
    return out


# ----------------------------------------------------------------- top-K
def topk_select(scores: torch.Tensor, n_state: Sequence[int], k: Sequence[int],
                state_begin: Sequence[int], seq_len: Sequence[int], n_alloc: int,
                bias_dtype: Optional[torch.dtype] = torch.bfloat16,
                want_topk_local: bool = False,
                keep_out: Optional[torch.Tensor] = None,
                bias_out: Optional[torch.Tensor] = None):
    """Top-k state tokens per request (score desc, index asc) and the kept positions.

    scores: fp32 (B, >= n_state[b]) with a contiguous last dim. k[b] is
    K_clamped. Returns (keep int64 (B, n_alloc), bias (B, n_alloc) in
    bias_dtype or None, topk_local int64 (B, max k) or None).
    """
    _require_cuda("scores", scores, torch.float32)
    if scores.dim() != 2 or scores.stride(1) != 1:
        raise ValueError("scores must be 2-D with a contiguous last dim")
    B = scores.shape[0]
    for name, arr in (("n_state", n_state), ("k", k), ("state_begin", state_begin), ("seq_len", seq_len)):
        if len(arr) != B:
            raise ValueError(f"{name} needs one entry per request")
    for b in range(B):
        if n_state[b] > scores.shape[1]:
            raise ValueError(f"request {b}: n_state {n_state[b]} exceeds the score row ({scores.shape[1]})")
    dev = scores.device
    keep = keep_out if keep_out is not None else torch.empty((B, n_alloc), dtype=torch.int64, device=dev)
    if keep.dtype != torch.int64 or keep.shape[0] != B or keep.shape[1] < n_alloc or keep.stride(1) != 1:
        raise ValueError("keep_out must be int64 (B, >= n_alloc) with a contiguous last dim")
    bias = None
    dt_code = 0
    if bias_dtype is not None or bias_out is not None:
        if bias_out is not None:
            bias = bias_out
        else:
            bias = torch.empty((B, n_alloc), dtype=bias_dtype, device=dev)
        if bias.dtype not in (torch.float32, torch.bfloat16) or bias.stride(1) != 1:
            raise ValueError("bias must be fp32 or bf16 with a contiguous last dim")
        dt_code = 0 if bias.dtype == torch.float32 else 1
    tl = None
    if want_topk_local:
        tl = torch.empty((B, max(int(x) for x in k)), dtype=torch.int64, device=dev)
    L = _lib.lib()
    with _device_ctx(scores):
        _lib.check_launch(L.tg_topk_select(
            scores.data_ptr(), scores.stride(0), B, _i32_array(n_state), _i32_array(k),
            _i32_array(state_begin), _i32_array(seq_len), int(n_alloc),
            keep.data_ptr(), keep.stride(0),
            bias.data_ptr() if bias is not None else None, bias.stride(0) if bias is not None else 0,
            dt_code, tl.data_ptr() if tl is not None else None, tl.stride(0) if tl is not None else 0,
            _stream(scores)))
    return keep, bias, tl


# ----------------------------------------------------------------- gather
def gather_spec_rows(src: torch.Tensor, dst: torch.Tensor, row_dim: int) -> _lib.GatherTensor:
    """Describe a gather of src -> dst along `row_dim` (batch is dim 0).

    The bytes of one row must be one contiguous block, or one contiguous
    block per index of the dims between the batch and the row dim (e.g. a
    (B, H, S, D) tensor gathered along S: one 256-byte segment per head).
    """
    if src.dtype != dst.dtype or src.device != dst.device:
        raise ValueError("src and dst must share dtype and device")
    if src.dim() != dst.dim() or src.dim() < 2:
        raise ValueError("src and dst must have the same rank (>= 2)")
    if not (1 <= row_dim < src.dim()):
        raise ValueError("row_dim must be a non-batch dim")
    es = src.element_size()
    inner_src = src.shape[row_dim + 1:]
    if tuple(dst.shape[row_dim + 1:]) != tuple(inner_src) or tuple(dst.shape[1:row_dim]) != tuple(src.shape[1:row_dim]):
        raise ValueError(f"src {tuple(src.shape)} and dst {tuple(dst.shape)} differ outside the row dim")

    def inner_block(t):
        # the dims after row_dim must be contiguous (one block per segment)
        expected = 1
        for d in range(t.dim() - 1, row_dim, -1):
            if t.shape[d] != 1 and t.stride(d) != expected:
                raise ValueError("the dims after the row dim must be contiguous")
            expected *= t.shape[d]
        return expected

    seg_elems = inner_block(src)
    inner_block(dst)
    mid = list(range(1, row_dim))
    n_seg = 1
    seg_stride_src = seg_stride_dst = 0
    if mid:
        if len(mid) > 1:
            raise ValueError("at most one dim between the batch and the row dim")
        n_seg = src.shape[mid[0]]
        seg_stride_src = src.stride(mid[0]) * es
        seg_stride_dst = dst.stride(mid[0]) * es
    g = _lib.GatherTensor()
    g.src = src.data_ptr()
    g.dst = dst.data_ptr()
    g.src_batch_stride = src.stride(0) * es
    g.src_row_stride = src.stride(row_dim) * es
    g.src_seg_stride = seg_stride_src
    g.dst_batch_stride = dst.stride(0) * es
    g.dst_row_stride = dst.stride(row_dim) * es
    g.dst_seg_stride = seg_stride_dst
    g.seg_bytes = seg_elems * es
    g.n_seg = n_seg
    g.reserved = 0
    return g


def gather_rows(specs: Sequence[_lib.GatherTensor], idx: torch.Tensor, n_valid: Sequence[int],
                n_rows: int, device: torch.device) -> None:
    """One launch: for every spec, dst row r <- src row idx[b, r] (r < n_valid[b]), zeros past it."""
    _require_cuda("idx", idx, torch.int64)
    if idx.dim() != 2 or idx.stride(1) != 1 or idx.shape[1] < n_rows:
        raise ValueError("idx must be int64 (B, >= n_rows) with a contiguous last dim")
    B = idx.shape[0]
    if len(n_valid) != B:
        raise ValueError("n_valid needs one entry per request")
    n = len(specs)
    if not 1 <= n <= _lib.MAX_GATHER_TENSORS:
        raise ValueError(f"1..{_lib.MAX_GATHER_TENSORS} tensors per launch, got {n}")
    arr = (_lib.GatherTensor * n)(*specs)
    L = _lib.lib()
    with _device_ctx(idx):
        _lib.check_launch(L.tg_gather_rows(arr, n, idx.data_ptr(), idx.stride(0), B, int(n_rows),
                                    _i32_array(n_valid), _stream(idx)))


# ----------------------------------------------------------------- layer glue
def _rows2d(name, t):
    if t.dim() < 2 or t.stride(-1) != 1:
        raise ValueError(f"{name} must have a contiguous last dim")
    lead = t.shape[:-1]
    # every leading dim must collapse onto one row stride
    flat = t.reshape(-1, t.shape[-1]) if t.is_contiguous() else None
    if flat is None:
        if t.dim() != 2:
            raise ValueError(f"{name}: non-contiguous inputs must be 2-D (rows, hidden)")
        flat = t
    return flat, lead


def add_rmsnorm(h: torch.Tensor, delta: Optional[torch.Tensor], weight: Optional[torch.Tensor],
                eps: float, h_out: Optional[torch.Tensor] = None, want_x: bool = True):
    """h_out = bf16(h + delta) (if delta); x = bf16(w * bf16(h_out * rsqrt(mean(h_out^2) + eps))).

    Returns (h_out, x); h_out is h itself when delta is None. h_out may be h (in place).
    """
    _require_cuda("h", h, torch.bfloat16)
    hf, lead = _rows2d("h", h)
    H = hf.shape[1]
    d_ptr, d_ld = None, 0
    if delta is not None:
        _require_cuda("delta", delta, torch.bfloat16)
        if delta.shape != h.shape:
            raise ValueError("delta must match h")
        df, _ = _rows2d("delta", delta)
        d_ptr, d_ld = df.data_ptr(), df.stride(0)
        if h_out is None:
            h_out = torch.empty_like(h)
        hof, _ = _rows2d("h_out", h_out)
    else:
        h_out, hof = h, hf
    x = None
    x_ptr, x_ld, w_ptr = None, 0, None
    if want_x:
        _require_cuda("weight", weight, torch.bfloat16)
        x = torch.empty(h.shape, dtype=torch.bfloat16, device=h.device)
        x_ptr, x_ld, w_ptr = x.data_ptr(), H, weight.data_ptr()
    L = _lib.lib()
    with _device_ctx(h):
        _lib.check_launch(L.tg_add_rmsnorm(hf.data_ptr(), hf.stride(0), d_ptr, d_ld,
                                    hof.data_ptr() if delta is not None else None,
                                    hof.stride(0) if delta is not None else 0,
                                    x_ptr, x_ld, w_ptr, hf.shape[0], H, float(eps), _stream(h)))
    return h_out, x


def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
                 cos: torch.Tensor, sin: torch.Tensor, eps: float) -> None:
    """In place: RMS-norm + RoPE of every head of q (B, S, Hq, 128) and k (B, S, Hkv, 128).

    Heads must be contiguous 128-element rows; cos/sin: (B, S, 128) bf16 (the
    rotary embedding of the rows' positions).
    """
    for nm, t in (("q", q), ("k", k)):
        _require_cuda(nm, t, torch.bfloat16)
        if t.dim() != 4 or t.shape[-1] != 128 or t.stride(-1) != 1 or t.stride(-2) != 128:
            raise ValueError(f"{nm} must be (B, S, heads, 128) with contiguous heads")
        # rows are addressed as (b * S + s) * row stride: the batch stride
        # matters only with more than one batch entry
        if t.shape[0] > 1 and t.stride(0) != t.shape[1] * t.stride(1):
            raise ValueError(f"{nm} rows must be evenly strided across the batch")
    B, S = q.shape[0], q.shape[1]
    if k.shape[:2] != q.shape[:2]:
        raise ValueError("q and k must cover the same rows")
    for nm, t in (("cos", cos), ("sin", sin)):
        _require_cuda(nm, t, torch.bfloat16)
        if t.shape != (B, S, 128) or t.stride(-1) != 1:
            raise ValueError(f"{nm} must be (B, S, 128) with a contiguous last dim")
    if cos.stride() != sin.stride():
        raise ValueError("cos and sin must share strides")
    L = _lib.lib()
    with _device_ctx(q):
        _lib.check_launch(L.tg_qk_norm_rope(q.data_ptr(), q.stride(1), q.shape[2], k.data_ptr(), k.stride(1),
                                     k.shape[2], B * S, S, q_norm_w.data_ptr(), k_norm_w.data_ptr(),
                                     cos.data_ptr(), sin.data_ptr(), cos.stride(0), cos.stride(1), 128,
                                     float(eps), _stream(q)))


def qk_norm_rope_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm_w: torch.Tensor,
                        k_norm_w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, eps: float,
                        k_cache: torch.Tensor, v_cache: torch.Tensor, slot: torch.Tensor) -> None:
    """qk_norm_rope for one decode token per row, appending it to the caches.

    q (B, 1, Hq, 128), k / v (B, 1, Hkv, 128) with contiguous heads; cos/sin
    (B, 1, 128); k_cache / v_cache (B, cap, Hkv, 128) contiguous; slot: an
    int64 (1,) device tensor, the cache slot the token goes to. q and k are
    normalised and rotated in place; the finished k and the v rows are also
    written to the caches (tg_qk_norm_rope_append)."""
    for nm, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(nm, t, torch.bfloat16)
        if t.dim() != 4 or t.shape[1] != 1 or t.shape[-1] != 128 or t.stride(-1) != 1 or t.stride(-2) != 128:
            raise ValueError(f"{nm} must be (B, 1, heads, 128) with contiguous heads")
    B = q.shape[0]
    if k.shape != v.shape or k.shape[0] != B:
        raise ValueError("k and v must be (B, 1, Hkv, 128)")
    for nm, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        _require_cuda(nm, t, torch.bfloat16)
        if t.dim() != 4 or t.shape[0] != B or t.shape[2:] != k.shape[2:] or not t.is_contiguous():
            raise ValueError(f"{nm} must be a contiguous (B, cap, Hkv, 128) tensor")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must have one shape")
    _require_cuda("slot", slot, torch.int64)
    for nm, t in (("cos", cos), ("sin", sin)):
        _require_cuda(nm, t, torch.bfloat16)
        if t.shape != (B, 1, 128) or t.stride(-1) != 1:
            raise ValueError(f"{nm} must be (B, 1, 128) with a contiguous last dim")
    L = _lib.lib()
    with _device_ctx(q):
        _lib.check_launch(L.tg_qk_norm_rope_append(
            q.data_ptr(), q.stride(0), q.shape[2], k.data_ptr(), k.stride(0), k.shape[2],
            v.data_ptr(), v.stride(0), B, q_norm_w.data_ptr(), k_norm_w.data_ptr(),
            cos.data_ptr(), sin.data_ptr(), cos.stride(0), cos.stride(1), 128, float(eps),
            k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), slot.data_ptr(),
            _stream(q)))


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """gu (..., 2*I) = [gate | up] -> bf16(bf16(silu(gate)) * up) (..., I)."""
    _require_cuda("gu", gu, torch.bfloat16)
    gf, lead = _rows2d("gu", gu)
    inter = gf.shape[1] // 2
    out = torch.empty(*lead, inter, dtype=torch.bfloat16, device=gu.device)
    L = _lib.lib()
    with _device_ctx(gu):
        _lib.check_launch(L.tg_silu_mul(gf.data_ptr(), gf.stride(0), out.data_ptr(), inter, gf.shape[0], inter,
                                 _stream(gu)))
    return out


def gemm_swiglu(x: torch.Tensor, w_gu: torch.Tensor, inter: int) -> torch.Tensor:
    """x (..., K), w_gu (2*inter, K) = [W_gate; W_up] -> bf16(bf16(silu(x W_gate^T)) * bf16(x W_up^T)),
    shape (..., inter): Qwen3MLP's act_fn(gate_proj(x)) * up_proj(x) as one tcgen05 GEMM with the
    SwiGLU in its epilogue (the [gate | up] projection never reaches HBM)."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("w_gu", w_gu, torch.bfloat16)
    xf, lead = _rows2d("x", x)
    if w_gu.dim() != 2 or w_gu.stride(1) != 1 or w_gu.shape[0] != 2 * inter or w_gu.shape[1] != xf.shape[1]:
        raise ValueError(f"w_gu must be (2*inter, K) = ({2 * inter}, {xf.shape[1]}) with a contiguous last dim")
    out = torch.empty(*lead, inter, dtype=torch.bfloat16, device=x.device)
    L = _lib.lib()
    with _device_ctx(x):
        _lib.check_launch(L.tg_gemm_swiglu(xf.data_ptr(), xf.stride(0), w_gu.data_ptr(), w_gu.stride(0),
                                           out.data_ptr(), inter, xf.shape[0], xf.shape[1], inter, _stream(x)))
    return out


def gemm_swiglu_readout(x: torch.Tensor, w_gu: torch.Tensor, w_readout: torch.Tensor,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The finalized gate's scoring branch fused into one tcgen05 GEMM: x (M, K) rows, w_gu
    (2*inter, K) = [W_gate; W_up], w_readout (inter,) -> fp32 scores (M,) =
    bf16(sum_c bf16(bf16(silu(G[:, c])) * U[:, c]) * w_readout[c]) with [G | U] the bf16 projection,
    silu with IEEE operations only. The [gate | up] projection never reaches memory; the partial
    dots go through an (inter/64, M) fp32 workspace allocated here."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("w_gu", w_gu, torch.bfloat16)
    _require_cuda("w_readout", w_readout, torch.bfloat16)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be (M, K) with a contiguous last dim")
    M, K = x.shape
    if w_readout.dim() != 1 or not w_readout.is_contiguous():
        raise ValueError("w_readout must be a contiguous vector")
    inter = w_readout.shape[0]
    if w_gu.dim() != 2 or w_gu.stride(1) != 1 or w_gu.shape != (2 * inter, K):
        raise ValueError(f"w_gu must be (2*inter, K) = ({2 * inter}, {K}) with a contiguous last dim")
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=x.device)
    else:
        _require_cuda("out", out, torch.float32)
        if out.dim() != 1 or out.shape[0] < M or out.stride(0) != 1:
            raise ValueError("out must be a contiguous fp32 vector of >= M entries")
    part = torch.empty((max(inter // 64, 1), max(M, 1)), dtype=torch.float32, device=x.device)
    L = _lib.lib()
    with _device_ctx(x):
        _lib.check_launch(L.tg_gemm_swiglu_readout(x.data_ptr(), x.stride(0), w_gu.data_ptr(), w_gu.stride(0),
                                                   w_readout.data_ptr(), part.data_ptr(), out.data_ptr(), M, K,
                                                   inter, _stream(x)))
    return out


def gemm_qkv_rope(x: torch.Tensor, w_qkv: torch.Tensor, n_q: int, n_k: int, q_norm_w: torch.Tensor,
                  k_norm_w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, eps: float) -> torch.Tensor:
    """x (B, S, K), w_qkv ((n_q + 2*n_k)*128, K) = [W_q; W_k; W_v] -> (B, S, n_q + 2*n_k, 128): the
    projection with every q and k head RMS-normalised (q_norm_w / k_norm_w) and rotated by cos / sin
    (B, S, 128) bf16, the v heads as projected: q_norm(q_proj(x)), k_norm(k_proj(x)) with RoPE and
    v_proj(x) as one tcgen05 GEMM with the norms and rotation in its epilogue."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("w_qkv", w_qkv, torch.bfloat16)
    if x.dim() != 3:
        raise ValueError("x must be (B, S, K)")
    B, S, K = x.shape
    if x.stride(2) != 1 or (B > 1 and x.stride(0) != S * x.stride(1)):
        raise ValueError("x rows must have a contiguous last dim and be evenly strided across the batch")
    xf = x.as_strided((B * S, K), (x.stride(1), 1))
    nh = n_q + 2 * n_k
    if w_qkv.dim() != 2 or w_qkv.stride(1) != 1 or w_qkv.shape != (nh * 128, K):
        raise ValueError(f"w_qkv must be ({nh * 128}, {K}) with a contiguous last dim")
    for nm, t in (("q_norm_w", q_norm_w), ("k_norm_w", k_norm_w)):
        _require_cuda(nm, t, torch.bfloat16)
        if t.shape != (128,) or not t.is_contiguous():
            raise ValueError(f"{nm} must be a contiguous (128,) tensor")
    for nm, t in (("cos", cos), ("sin", sin)):
        _require_cuda(nm, t, torch.bfloat16)
        if t.shape != (B, S, 128) or t.stride(-1) != 1:
            raise ValueError(f"{nm} must be (B, S, 128) with a contiguous last dim")
    if cos.stride() != sin.stride():
        raise ValueError("cos and sin must share strides")
    out = torch.empty(B, S, nh, 128, dtype=torch.bfloat16, device=x.device)
    L = _lib.lib()
    with _device_ctx(x):
        _lib.check_launch(L.tg_gemm_qkv_rope(xf.data_ptr(), xf.stride(0), w_qkv.data_ptr(), w_qkv.stride(0),
                                             out.data_ptr(), nh * 128, B * S, K, n_q, n_k, q_norm_w.data_ptr(),
                                             k_norm_w.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
                                             cos.stride(1), S, float(eps), _stream(x)))
    return out


def device_error(clear: bool = False) -> int:
    """Flags recorded by kernels whose bounded waits gave up on the current device (synchronises)."""
    return _lib.device_error(torch.cuda.current_stream().cuda_stream, clear)


# ----------------------------------------------------------------- finalized gate
def branch_score(gu: torch.Tensor, w_row: torch.Tensor, row_begin: Sequence[int],
                 row_count: Sequence[int], out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Readout of the finalized gate's scoring branch over the fused [gate | up] rows.

    scores[b, r] = bf16(sum_k bf16(bf16(silu(g_k)) * u_k) * w_row[k]) (as fp32, -0 -> +0)
    with [g | u] = gu[b, row_begin[b] + r, :2*inter], for r < row_count[b].
    gu: (B, S, >= 2*inter) bf16 with a contiguous last dim; w_row: (inter,) bf16.
    Returns fp32 (B, max(row_count)); entries past row_count[b] untouched
    (zero when allocated here).
    """
    _require_cuda("gu", gu, torch.bfloat16)
    _require_cuda("w_row", w_row, torch.bfloat16)
    if gu.dim() != 3 or gu.stride(-1) != 1:
        raise ValueError("gu must be (B, S, 2*inter) with a contiguous last dim")
    if w_row.dim() != 1 or not w_row.is_contiguous():
        raise ValueError("w_row must be a contiguous vector")
    B, S, W = gu.shape
    inter = w_row.shape[0]
    if W < 2 * inter:
        raise ValueError(f"gu rows hold {W} values, need [gate | up] = {2 * inter}")
    if len(row_begin) != B or len(row_count) != B:
        raise ValueError("row_begin / row_count need one entry per request")
    for b in range(B):
        if row_begin[b] < 0 or row_count[b] < 0 or row_begin[b] + row_count[b] > S:
            raise ValueError(f"request {b}: rows [{row_begin[b]}, {row_begin[b] + row_count[b]}) "
                             f"outside [0, {S})")
    n_max = max(int(c) for c in row_count)
    if out is None:
        out = torch.zeros((B, max(n_max, 1)), dtype=torch.float32, device=gu.device)
    else:
        _require_cuda("out", out, torch.float32)
        if out.dim() != 2 or out.shape[0] != B or out.shape[1] < n_max or out.stride(1) != 1:
            raise ValueError("out must be (B, >= max(row_count)) fp32 with a contiguous last dim")
    L = _lib.lib()
    with _device_ctx(gu):
        _lib.check_launch(L.tg_branch_score(gu.data_ptr(), gu.stride(0), gu.stride(1), inter, w_row.data_ptr(),
                                     B, _i32_array(row_begin), _i32_array(row_count), out.data_ptr(),
                                     out.stride(0), _stream(gu)))
    return out


def phase2_tables(scores: torch.Tensor, state_begin: Sequence[int], n_state: Sequence[int],
                  keep: torch.Tensor, n_kept: Sequence[int], gate_scale: torch.Tensor,
                  attn_scale: torch.Tensor, eps: float, gain: float = 1.0):
    """Per-layer Phase-2 key bias and query scale of the finalized gate.

    scores: raw branch scores fp32 (B, >= n_state[b]); keep: int64 (B, n_alloc)
    kept positions; gate_scale / attn_scale: effective (softplus-applied)
    (L', H) fp32. Returns (bias, q_scale), each fp32 (L', B, H, n_alloc):
    layer l's slice is the (B, H, S) bias / q_row_scale of keybias_attention.
    """
    _require_cuda("scores", scores, torch.float32)
    _require_cuda("keep", keep, torch.int64)
    _require_cuda("gate_scale", gate_scale, torch.float32)
    _require_cuda("attn_scale", attn_scale, torch.float32)
    if scores.dim() != 2 or scores.stride(1) != 1:
        raise ValueError("scores must be 2-D with a contiguous last dim")
    if keep.dim() != 2 or keep.stride(1) != 1:
        raise ValueError("keep must be 2-D with a contiguous last dim")
    if gate_scale.dim() != 2 or gate_scale.shape != attn_scale.shape:
        raise ValueError("gate_scale and attn_scale must both be (L', H)")
    B, n_alloc = keep.shape
    if scores.shape[0] != B:
        raise ValueError("one score row per request")
    for name, arr in (("state_begin", state_begin), ("n_state", n_state), ("n_kept", n_kept)):
        if len(arr) != B:
            raise ValueError(f"{name} needs one entry per request")
    for b in range(B):
        if n_state[b] > scores.shape[1]:
            raise ValueError(f"request {b}: n_state {n_state[b]} exceeds the score row ({scores.shape[1]})")
    Lp, H = gate_scale.shape
    gs = gate_scale.contiguous()
    at = attn_scale.contiguous()
    bias = torch.empty((Lp, B, H, n_alloc), dtype=torch.float32, device=scores.device)
    q_scale = torch.empty_like(bias)
    L = _lib.lib()
    with _device_ctx(scores):
        _lib.check_launch(L.tg_phase2_tables(scores.data_ptr(), scores.stride(0), B, _i32_array(state_begin),
                                      _i32_array(n_state), keep.data_ptr(), keep.stride(0),
                                      _i32_array(n_kept), int(n_alloc), gs.data_ptr(), at.data_ptr(),
                                      int(Lp), int(H), float(eps), float(gain), bias.data_ptr(),
                                      q_scale.data_ptr(), _stream(scores)))
    return bias, q_scale


# ----------------------------------------------------------------- decode attention
def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, n_valid: torch.Tensor,
                     n_prefix: int, n_keys: int, bias: Optional[torch.Tensor] = None,
                     q_scale: Optional[torch.Tensor] = None,
                     softmax_scale: Optional[float] = None,
                     out: Optional[torch.Tensor] = None,
                     n_keys_dev: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One decode query per (row, head) against a gated KV cache (tg_decode_attn).

    q: (B, Hq, 128) bf16; k, v: (B, cap, Hkv, 128) bf16 caches holding the
    prefix (kept tokens, or the full Phase-1 cache) in [0, n_prefix) and the
    decoded tokens in [n_prefix, n_keys); n_valid: (B,) int32 on the device,
    prefix keys valid per row (the rest are pad slots, masked). bias: fp32
    broadcastable to (B, Hq, n_prefix) with a contiguous last dim, added to
    the prefix keys' scores (score units); q_scale: fp32 (B, Hq), the
    per-step query scale (q <- bf16(q * bf16(q_scale))). n_keys_dev: an int32
    (1,) device tensor holding the keys to attend (at most n_keys, which then
    only bounds the launch): the form a captured CUDA graph replays while the
    cache grows (tg_decode_attn_ex). Returns (B, Hq, 128) bf16.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t, torch.bfloat16)
        if t.stride(-1) != 1:
            raise ValueError(f"{name} must have a contiguous last dim")
    if q.dim() != 3 or k.dim() != 4 or v.shape != k.shape:
        raise ValueError(f"shapes: q {tuple(q.shape)} (B, Hq, D), k/v {tuple(k.shape)} (B, cap, Hkv, D)")
    B, Hq, D = q.shape
    cap, Hkv = k.shape[1], k.shape[2]
    if k.shape[0] != B or k.shape[3] != D:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)} k {tuple(k.shape)}")
    if not 0 <= n_prefix <= n_keys <= cap:
        raise ValueError(f"need 0 <= n_prefix ({n_prefix}) <= n_keys ({n_keys}) <= cache capacity ({cap})")
    _require_cuda("n_valid", n_valid, torch.int32)
    if n_valid.numel() != B or not n_valid.is_contiguous():
        raise ValueError("n_valid must be a contiguous (B,) int32 tensor")
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=q.device)
    bias_ptr, bsb, bsh = None, 0, 0
    if bias is not None:
        _require_cuda("bias", bias, torch.float32)
        bb = bias
        while bb.dim() < 3:
            bb = bb.unsqueeze(0)
        if bb.shape[-1] < n_prefix or bb.stride(-1) != 1 or bb.shape[0] not in (1, B) \
                or bb.shape[1] not in (1, Hq):
            raise ValueError(f"bias {tuple(bias.shape)} must broadcast to ({B}, {Hq}, >= {n_prefix}) "
                             "with a contiguous last dim")
        bsb = 0 if bb.shape[0] == 1 else bb.stride(0)
        bsh = 0 if bb.shape[1] == 1 else bb.stride(1)
        bias_ptr = bb.data_ptr()
    qs_ptr, qsb = None, 0
    if q_scale is not None:
        _require_cuda("q_scale", q_scale, torch.float32)
        if q_scale.shape != (B, Hq) or q_scale.stride(1) != 1:
            raise ValueError(f"q_scale must be (B, Hq) = ({B}, {Hq}) with a contiguous last dim")
        qs_ptr, qsb = q_scale.data_ptr(), q_scale.stride(0)
    L = _lib.lib()
    with _device_ctx(q):
        nbytes = ctypes.c_size_t(0)
        _lib.check(L.tg_decode_attn_workspace(B, Hq, int(n_keys), ctypes.byref(nbytes)))
        ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device) if nbytes.value else None
        if n_keys_dev is not None:
            _require_cuda("n_keys_dev", n_keys_dev, torch.int32)
        _lib.check_launch(L.tg_decode_attn_ex(
            q.data_ptr(), q.stride(0), q.stride(1), qs_ptr, qsb,
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
            v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
            bias_ptr, bsb, bsh, n_valid.data_ptr(), int(n_prefix), int(n_keys),
            n_keys_dev.data_ptr() if n_keys_dev is not None else None,
            out.data_ptr(), out.stride(0), out.stride(1),
            ws.data_ptr() if ws is not None else None, nbytes.value,
            B, Hq, Hkv, D, float(softmax_scale), _stream(q)))
    return out


# ----------------------------------------------------------------- decode projections
def gemv(x: torch.Tensor, w: torch.Tensor, swiglu: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ w.T for the decode step's few rows (tg_gemv): x (B, K) bf16 with
    B <= 8 and K a multiple of 256, w (N, K) bf16 (row-major, contiguous
    rows). swiglu: w is the fused [gate; up] weight (2I, K) and the result is
    bf16(bf16(silu(gate)) * up), (B, I)."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("w", w, torch.bfloat16)
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1] or x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError(f"x {tuple(x.shape)} (B, K) and w {tuple(w.shape)} (N, K) with contiguous rows")
    B, K = x.shape
    N = w.shape[0] // 2 if swiglu else w.shape[0]
    if swiglu and w.shape[0] % 2:
        raise ValueError("the fused [gate; up] weight has an even number of rows")
    if out is None:
        out = torch.empty((B, N), dtype=torch.bfloat16, device=x.device)
    L = _lib.lib()
    with _device_ctx(x):
        _lib.check_launch(L.tg_gemv(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
                             B, N, K, int(bool(swiglu)), _stream(x)))
    return out
