"""The gate served by the B200 scorer: a 1-wide fp32 linear readout + log-sigmoid.

The reference scores the state span with `gate(h_art.to(gate dtype))` and
selects on `gate.aggregate(scores)` (tokengate/e2e_gate/gate_module/
gate_forward.py:1396-1412). The benchmarked synthetic gate is a 2048 -> 1 linear
map with log-sigmoid, i.e. the reference's DeterministicGate fixture
(tests/inference/test_prefill_memory.py:18-33: fp32 readout, n_layers_bias=0,
selection_mode "topk", identity aggregate) with log-sigmoid applied.
`LinLogSigGate` is that module; `readout_vector` extracts the weights the
kernel consumes and rejects gates the kernel does not serve (scoring branch,
per-head/per-layer outputs, threshold or random selection).
"""
import torch


class LinLogSigGate(torch.nn.Module):
    """score(h) = logsigmoid(w . h), fp32 parameters; selection by top-K."""

    n_layers_bias = 0
    selection_mode = "topk"
    random_topk = False
    gate_branch = None

    def __init__(self, hidden_size: int, std: float = None, generator: torch.Generator = None):
        super().__init__()
        self.readout = torch.nn.Linear(hidden_size, 1, bias=False, dtype=torch.float32)
        std = hidden_size ** -0.5 if std is None else std
        with torch.no_grad():
            self.readout.weight.copy_(torch.randn(1, hidden_size, generator=generator) * std)

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        return torch.nn.functional.logsigmoid(self.readout(hidden)).squeeze(-1)

    def aggregate(self, scores: torch.Tensor) -> torch.Tensor:
        return scores


def readout_vector(gate, hidden_size: int, device) -> torch.Tensor:
    """The (hidden_size,) fp32 weight vector of a gate the B200 scorer serves."""
    if getattr(gate, "gate_branch", None) is not None:
        raise NotImplementedError("gates with a scoring branch (LN2 -> SwiGLU -> readout) are not "
                                  "served by the B200 scorer yet")
    if getattr(gate, "selection_mode", "topk") != "topk" or getattr(gate, "random_topk", False):
        raise NotImplementedError("only top-K selection is served by the B200 selection kernel")
    if getattr(gate, "n_layers_bias", 0) != 0:
        raise NotImplementedError("per-layer gate scales (n_layers_bias > 0) are not served")
    ro = getattr(gate, "readout", None)
    if not isinstance(ro, torch.nn.Linear) or ro.out_features != 1 or ro.bias is not None:
        raise NotImplementedError("the gate must expose a bias-free 1-wide `readout` Linear")
    w = ro.weight.detach().reshape(-1)
    if w.numel() != hidden_size:
        raise ValueError(f"gate readout has {w.numel()} inputs, model hidden size is {hidden_size}")
    # cached per device and weight version: a CPU-resident gate would otherwise
    # cost a pageable host-to-device copy (a stream synchronisation) per prefill
    key = (str(device), w.data_ptr(), ro.weight._version)
    cached = getattr(gate, "_tg_readout", None)
    if cached is None or cached[0] != key:
        cached = (key, w.to(device=device, dtype=torch.float32).contiguous())
        gate._tg_readout = cached
    return cached[1]


# ----------------------------------------------------------------------------
# The finalized TokenGate gate (tokengate/e2e_gate/gate_module/e2e_gate_module.py)
# ----------------------------------------------------------------------------
import math

import torch.nn.functional as F

_RMS_EPS = 1e-6          # e2e_gate_module.py:74
SYNTHETIC_E2E_SEED = 20261012


class CastLinear(torch.nn.Module):
    """fp32 parameter storage, matmul in the input's dtype; nn.Linear state-dict
    keys (e2e_gate_module.py:89-135)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = torch.nn.Parameter(torch.zeros(out_features, in_features, dtype=torch.float32,
                                                     device=device))
        if bias:
            self.bias = torch.nn.Parameter(torch.zeros(out_features, dtype=torch.float32, device=device))
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b = None if self.bias is None else self.bias.to(x.dtype)
        return F.linear(x, self.weight.to(x.dtype), b)


class BranchMLP(torch.nn.Module):
    """The scoring branch: a SwiGLU clone of the gate layer's MLP whose down_proj
    is the absorbed readout row (1, inter) (Qwen3MLP as load_gate rebuilds it,
    e2e_gate_module.py:495-516)."""

    def __init__(self, d_model: int, inter: int, out_features: int = 1, device=None):
        super().__init__()
        self.gate_proj = CastLinear(d_model, inter, device=device)
        self.up_proj = CastLinear(d_model, inter, device=device)
        self.down_proj = CastLinear(inter, out_features, device=device)

    def forward(self, z: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(z)) * self.up_proj(z))


class E2EGate(torch.nn.Module):
    """The finalized gate: absorbed shared readout + sequence RMSNorm + softplus
    scales (e2e_gate_module.py:204-400), with the same parameter names, buffers
    and state-dict keys, so reference checkpoints load unchanged."""

    normed_gate = True
    softplus_gate_scale = True
    scaled_softmax_scale = True
    use_attn_scale = True
    shared_readout = True
    absorbed_readout = True
    readout_residual = False
    gate_branch_mode = "mlp"
    per_layer_gate = True
    learnable_sss_scale = True
    head_agg = "avg"
    ste_factor = 0.0
    random_topk = False

    def __init__(self, d_model: int, n_heads: int = 1, n_layers_bias: int = 0,
                 selection_mode: str = "topk", tau: float = 0.5):
        super().__init__()
        if selection_mode not in ("topk", "threshold"):
            raise ValueError(f"selection_mode must be 'topk' or 'threshold', got {selection_mode!r}")
        if n_layers_bias <= 0:
            raise ValueError("n_layers_bias must be > 0: the finalized gate scales its bias per "
                             "Phase-2 (layer, head)")
        from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_layers_bias = n_layers_bias
        self.selection_mode = selection_mode
        self.tau = float(tau)
        self.gate_branch = None
        if n_heads > 1:
            self.register_buffer("agg_weights", torch.full((n_heads,), 1.0 / n_heads))
        self.gate_scale = torch.nn.Parameter(torch.zeros(n_layers_bias, n_heads))
        self.attn_scale = torch.nn.Parameter(torch.full((n_layers_bias, n_heads),
                                                        math.log(math.expm1(1.0))))
        self.b_norm = Qwen3RMSNorm(1, eps=_RMS_EPS)
        self.b_norm.weight.requires_grad_(False)

    def attn_scale_eff(self) -> torch.Tensor:
        return F.softplus(self.attn_scale)

    @torch.no_grad()
    def set_qk_norm_scales(self, model: torch.nn.Module, gate_layer: int) -> list:
        """gate_scale raw = softplus^-1(||g_q * g_k||_2 / sqrt(head_dim)) of each
        Phase-2 layer's q/k norm gains, broadcast over heads (:281-319)."""
        layers = model.model.layers
        idxs = list(range(gate_layer + 1, len(layers)))
        if len(idxs) != self.n_layers_bias:
            raise ValueError(f"n_layers_bias={self.n_layers_bias} != phase-2 layer count {len(idxs)}")
        vals = []
        for row, li in enumerate(idxs):
            attn = layers[li].self_attn
            gq = attn.q_norm.weight.detach().float()
            gk = attn.k_norm.weight.detach().float()
            s_l = float((gq * gk).norm() / math.sqrt(gq.numel()))
            self.gate_scale.data[row].fill_(math.log(math.expm1(s_l)))
            vals.append(s_l)
        return vals

    def forward(self, scores: torch.Tensor) -> torch.Tensor:
        """(n_art, 1) raw branch scores -> (n_art, L', H) Phase-2 bias (:348-385)."""
        gs = F.softplus(self.gate_scale)
        b = scores.view(*scores.shape[:-1], 1, 1).expand(*scores.shape[:-1], self.n_layers_bias,
                                                          self.n_heads)
        bn = self.b_norm(b.movedim(-3, -1)).movedim(-1, -3)
        return bn * gs

    def aggregate(self, b: torch.Tensor) -> torch.Tensor:
        """Selection score: the first Phase-2 layer's slot, mean over heads (:387-399)."""
        if b.dim() == 3:
            b = b[:, 0, :]
        if self.n_heads == 1:
            return b
        return (b * self.agg_weights).sum(-1)


_FINALIZED_FLAGS = (
    ("n_input_layers", 1, 1), ("score_source", "hidden", "hidden"), ("learned_agg", False, False),
    ("tanh_gate", False, False), ("qk_norm_scale", False, False), ("softplus_sss", False, False),
    ("sss_frozen_gate_scale", False, False), ("ste_factor", 0.0, 0.0), ("normed_gate", True, True),
    ("use_attn_scale", True, True), ("scaled_softmax_scale", True, True),
    ("softplus_gate_scale", True, True), ("shared_readout", True, True),
    ("absorbed_readout", True, True), ("readout_residual", False, False),
    ("gate_branch_mode", "mlp", "mlp"), ("head_agg", "avg", "avg"), ("per_layer_gate", True, True),
    ("learnable_sss_scale", True, True),
)


def save_gate(gate: E2EGate, path: str, metadata: dict = None) -> None:
    """Write the reference's gate checkpoint format (e2e_gate_module.py:402-431)."""
    obj = {"state_dict": gate.state_dict(), "d_model": gate.d_model, "n_heads": gate.n_heads,
           "n_layers_bias": gate.n_layers_bias, "selection_mode": gate.selection_mode, "tau": gate.tau}
    for key, expected, _default in _FINALIZED_FLAGS:
        if key in ("n_input_layers", "score_source", "learned_agg", "tanh_gate", "qk_norm_scale",
                   "softplus_sss", "sss_frozen_gate_scale"):
            continue
        obj[key] = expected
    obj["metadata"] = metadata or {}
    torch.save(obj, path)


def load_gate(path, trusted: bool = False):
    """Load a reference gate checkpoint -> (E2EGate, metadata) (e2e_gate_module.py:434-526).

    Validates the finalized-architecture flags, rebuilds the scoring branch from
    the saved shapes (down_proj (1, inter): the absorbed readout) with fp32
    storage and loads the state dict strictly. The file is read with torch's
    weights-only unpickler unless `trusted` (the reference loads with full
    pickle; pass trusted=True for a checkpoint whose metadata holds other
    Python objects and whose origin you trust). `path` may also be the
    already-loaded checkpoint dict.
    """
    if isinstance(path, dict):
        obj = path
    else:
        obj = torch.load(path, map_location="cpu", weights_only=not trusted)

    for key, expected, default in _FINALIZED_FLAGS:
        got = obj.get(key, default)
        if got != expected:
            raise ValueError(f"checkpoint {path!r} has {key}={got!r}; the finalized gate requires "
                             f"{key}={expected!r}")
    gc = obj.get("gate_cond", "none")
    if gc not in ("none", None) or obj.get("use_boundary_cond", False):
        raise ValueError(f"checkpoint {path!r} uses gate_cond={gc!r}; only 'none' is supported")
    sd = dict(obj["state_dict"])
    if "post_proj.weight" in sd:
        raise ValueError(f"checkpoint {path!r} carries post_proj.weight (removed post-top-K projection)")
    gate = E2EGate(d_model=obj["d_model"], n_heads=obj.get("n_heads", 1),
                   n_layers_bias=obj.get("n_layers_bias", 0),
                   selection_mode=obj.get("selection_mode", "topk"), tau=obj.get("tau", 0.5))
    if not any(k.startswith("gate_branch.") for k in sd):
        raise ValueError(f"checkpoint {path!r} carries no gate_branch.* weights")
    inter, dm = sd["gate_branch.gate_proj.weight"].shape
    dp = sd.get("gate_branch.down_proj.weight")
    out = dp.shape[0] if dp is not None else dm
    gate.gate_branch = BranchMLP(dm, inter, out_features=out)
    for name in ("gate_proj", "up_proj", "down_proj"):
        if f"gate_branch.{name}.bias" in sd:
            lin = getattr(gate.gate_branch, name)
            setattr(gate.gate_branch, name, CastLinear(lin.in_features, lin.out_features, bias=True))
    missing, unexpected = gate.load_state_dict(sd, strict=False)
    if missing or unexpected:
        raise RuntimeError(f"load_gate({path!r}): state_dict mismatch: missing={missing}, "
                           f"unexpected={unexpected}")
    bad = [n for n, p in gate.gate_branch.named_parameters() if p.dtype != torch.float32]
    if bad:
        raise RuntimeError(f"load_gate({path!r}): scoring branch parameters must be fp32, got {bad}")
    return gate, obj.get("metadata", {})


@torch.no_grad()
def build_gate_branch(model: torch.nn.Module, gate: E2EGate, gate_layer: int) -> BranchMLP:
    """Attach the scoring branch: an fp32 clone of layer `gate_layer`'s MLP with
    the absorbed readout row zero-initialised (gate_forward.py:261-343)."""
    mlp = model.model.layers[gate_layer].mlp
    inter, dm = mlp.gate_proj.weight.shape
    dev = mlp.gate_proj.weight.device
    br = BranchMLP(dm, inter, out_features=1, device=dev)
    br.gate_proj.weight.copy_(mlp.gate_proj.weight.float())
    br.up_proj.weight.copy_(mlp.up_proj.weight.float())
    gate.gate_branch = br
    return br


@torch.no_grad()
def synthetic_e2e_gate(model: torch.nn.Module, gate_layer: int, seed: int = SYNTHETIC_E2E_SEED,
                       device=None) -> E2EGate:
    """A finalized gate for a model without a trained checkpoint, built the way
    the reference's own equivalence test builds one
    (tests/inference/test_bench_batched_equivalence.py:134-144): E2EGate over
    the Phase-2 layers and the model's query heads, set_qk_norm_scales,
    build_gate_branch, then a seeded readout row (std 0.05) and a seeded
    0.3-std perturbation of gate_scale and attn_scale so layers and heads
    differ."""
    cfg = model.config
    n_lb = cfg.num_hidden_layers - 1 - gate_layer
    dev = device if device is not None else next(model.parameters()).device
    gate = E2EGate(d_model=cfg.hidden_size, n_heads=cfg.num_attention_heads, n_layers_bias=n_lb)
    gate.set_qk_norm_scales(model, gate_layer)
    build_gate_branch(model, gate, gate_layer)
    gate = gate.to("cpu").float()
    g = torch.Generator().manual_seed(seed)
    dp = gate.gate_branch.down_proj.weight
    dp.copy_(torch.randn(dp.shape, generator=g) * 0.05)
    gate.gate_scale.add_(torch.randn(gate.gate_scale.shape, generator=g) * 0.3)
    gate.attn_scale.add_(torch.randn(gate.attn_scale.shape, generator=g) * 0.3)
    return gate.to(dev).eval()


class E2EKernelWeights:
    """The finalized gate's operands for the B200 kernels, derived once per gate
    state: the fused [gate; up] projection in bf16 (CastLinear's compute dtype),
    the readout row in bf16, softplus(gate_scale) and softplus(attn_scale) as
    fp32 (L', H) tables, the RMSNorm gain and eps."""

    def __init__(self, gate: E2EGate, device, dtype=torch.bfloat16):
        br = gate.gate_branch
        for name in ("gate_proj", "up_proj", "down_proj"):
            if getattr(br, name).bias is not None:
                raise NotImplementedError("scoring-branch biases are not served by the B200 readout")
        if br.down_proj.weight.shape[0] != 1:
            raise NotImplementedError("the scoring branch must end in the absorbed 1-row readout")
        with torch.no_grad():
            self.wgu = torch.cat([br.gate_proj.weight, br.up_proj.weight], 0).to(
                device=device, dtype=dtype).contiguous()
            self.w_row = br.down_proj.weight.reshape(-1).to(device=device, dtype=dtype).contiguous()
            self.gate_scale = F.softplus(gate.gate_scale.detach().to(device=device,
                                                                     dtype=torch.float32)).contiguous()
            self.attn_scale = F.softplus(gate.attn_scale.detach().to(device=device,
                                                                     dtype=torch.float32)).contiguous()
            self.gain = float(gate.b_norm.weight.detach().float().reshape(-1)[0])
            # all first-layer scales 0: every aggregate is 0 and the selection
            # falls back to index order
            self.degenerate = not bool((self.gate_scale[0] > 0).any())
        self.eps = float(gate.b_norm.variance_epsilon)
        self.inter = self.w_row.numel()
        self.n_heads = gate.n_heads
        self.n_layers_bias = gate.n_layers_bias


def e2e_kernel_weights(gate: E2EGate, device) -> E2EKernelWeights:
    """Cached E2EKernelWeights, rebuilt when a gate parameter changes."""
    key = (str(device),) + tuple((p.data_ptr(), p._version) for p in gate.parameters())
    cached = getattr(gate, "_tg_kernel_weights", None)
    if cached is None or cached[0] != key:
        cached = (key, E2EKernelWeights(gate, device))
        gate._tg_kernel_weights = cached
    return cached[1]


def is_e2e_gate(gate) -> bool:
    """True for a gate with a scoring branch (the finalized architecture)."""
    return getattr(gate, "gate_branch", None) is not None
