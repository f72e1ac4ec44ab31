"""The fused Phase-2 layer loop as one CUDA graph per (model, gate layer, batch, padded length).

Phase 2 runs every layer above the gate layer on the kept tokens. At small K
it is launch-bound: ~9 launches per layer, a few microseconds of GPU work
each. Here the loop of the fused path (tokengate_b200.layers) is captured
once per shape and replayed, so the host issues one launch. Mirrors the
reference's phase2_graph.replay_layers (tokengate/e2e_gate/gate_module/
phase2_graph.py:1-60, :170-230), including its contract:

  * exactness: the captured work is the same kernels on the same values; the
    inputs (kept hidden rows, RoPE tables of the kept positions, the key bias
    or the finalized gate's bias / query-scale tables) are copied into the
    graph's static buffers before each replay;
  * the K/V the returned cache holds are the graph's own buffers: the next
    replay of the same shape overwrites them, so a caller that decodes from
    the cache must be done with it (or clone it) before the next prefill of
    that shape;
  * shapes above GRAPH_MAX_TOKENS are not captured (they are compute-bound
    and usually unique); the caller pads the kept length to a bucket
    (set_phase2_bucket) so the set of shapes stays small.

Graphs are kept in a small LRU per process (MAX_GRAPHS) sharing one memory
pool; the head (final norm of each request's last kept row, lm_head) stays
outside the graph because its row indices change with n_kept.
"""
from collections import OrderedDict
from typing import Optional

import torch

from . import _lib, ops
from .layers import layer_forward, layer_mlp
from .model import PrefillCache, _CacheLayer

GRAPH_MAX_TOKENS = 10240
MAX_GRAPHS = 8

_GRAPHS: "OrderedDict[tuple, _Phase2Graph]" = OrderedDict()
_POOL = None
# library kernel launches replayed through graphs since import (each replay
# adds the count its capture recorded)
REPLAYED_LAUNCHES = 0


def _pool():
    global _POOL
    if _POOL is None:
        _POOL = torch.cuda.graph_pool_handle()
    return _POOL


def clear() -> None:
    """Drop every captured graph (and with them their static buffers)."""
    _GRAPHS.clear()


class _Phase2Graph:
    """Static buffers, the captured graph and the cache it writes."""

    def __init__(self, fw, gate_layer: int, n_layers: int, B: int, n_alloc: int, hidden: int,
                 bias_shape, qs_shape, split_gate_mlp: bool, device):
        self.fw, self.gate_layer, self.n_layers = fw, gate_layer, n_layers
        self.split = split_gate_mlp
        self.hs = torch.zeros(B, n_alloc, hidden, dtype=torch.bfloat16, device=device)
        self.cos = torch.zeros(B, n_alloc, fw[0].head_dim, dtype=torch.bfloat16, device=device)
        self.sin = torch.zeros_like(self.cos)
        self.bias = torch.zeros(bias_shape, dtype=torch.float32, device=device)
        self.qs = None if qs_shape is None else torch.ones(qs_shape, dtype=torch.float32, device=device)
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(2):  # first calls (library handles, kernel attributes) outside the capture
                self._run(PrefillCache(n_layers))
        torch.cuda.current_stream(device).wait_stream(side)
        self.cache = PrefillCache(n_layers)
        self.graph = torch.cuda.CUDAGraph()
        n0 = _lib.LAUNCH_CALLS
        with torch.cuda.graph(self.graph, pool=_pool(), stream=side):
            self.out_h, self.out_delta = self._run(self.cache)
        self.launches = _lib.LAUNCH_CALLS - n0   # library kernels per replay

    def _run(self, cache):
        fw, L = self.fw, self.gate_layer
        h = self.hs
        delta: Optional[torch.Tensor] = None
        if self.split:  # the gate layer's own MLP on the kept rows (finalized gate)
            _, x2 = ops.add_rmsnorm(h, None, fw[L].post_w, fw[L].eps)
            delta = layer_mlp(fw[L], x2)
        for i in range(L + 1, self.n_layers):
            li = i - L - 1
            if self.qs is not None:
                bias, qs = self.bias[li], self.qs[li]
            else:
                bias, qs = self.bias, None
            h, delta = layer_forward(fw[i], h, delta, self.cos, self.sin, cache, i, gate_bias=bias,
                                     q_row_scale=qs)
        return h, delta

    def replay(self, hs, cos, sin, bias, qs, cache):
        global REPLAYED_LAUNCHES
        REPLAYED_LAUNCHES += self.launches
        self.hs.copy_(hs)
        self.cos.copy_(cos)
        self.sin.copy_(sin)
        self.bias.copy_(bias)
        if self.qs is not None:
            self.qs.copy_(qs)
        self.graph.replay()
        for i in range(self.gate_layer + 1, self.n_layers):
            src = self.cache.layers[i]
            dst = _CacheLayer()
            dst.k_tok, dst.v_tok = src.k_tok, src.v_tok
            cache.layers[i] = dst
        return self.out_h, self.out_delta


def run_phase2(model, fw, gate_layer: int, hs_pruned: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               bias: torch.Tensor, qs: Optional[torch.Tensor], cache, split_gate_mlp: bool):
    """Phase 2 through a captured graph; returns (h, delta) of the last layer
    (the graph's output buffers), or None when the shape is not captured."""
    B, n_alloc, H = hs_pruned.shape
    if n_alloc > GRAPH_MAX_TOKENS:
        return None
    n_layers = len(model.model.layers)
    key = (id(model), gate_layer, B, n_alloc, tuple(bias.shape), None if qs is None else tuple(qs.shape),
           split_gate_mlp, hs_pruned.device.index)
    g = _GRAPHS.get(key)
    if g is None:
        if len(_GRAPHS) >= MAX_GRAPHS:
            _GRAPHS.popitem(last=False)
        g = _Phase2Graph(fw, gate_layer, n_layers, B, n_alloc, H, tuple(bias.shape),
                         None if qs is None else tuple(qs.shape), split_gate_mlp, hs_pruned.device)
        _GRAPHS[key] = g
    else:
        _GRAPHS.move_to_end(key)
    return g.replay(hs_pruned, cos, sin, bias, qs, cache)
