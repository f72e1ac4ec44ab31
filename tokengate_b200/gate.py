"""The gate served by the B200 scorer: a 1-wide fp32 linear readout + log-sigmoid.

The reference scores the state span with `gate(h_art.to(gate dtype))` and
selects on `gate.aggregate(scores)` (tokengate/e2e_gate/gate_module/
gate_forward.py:1396-1412). BASELINE's synthetic gate is a 2048 -> 1 linear
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
    return w.to(device=device, dtype=torch.float32).contiguous()
