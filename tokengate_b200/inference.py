"""Public API: load_model(...) -> TokenGateModel; model.generate(ids, tok, max_kept_prefill_tokens=K).

Mirrors the reference API (tokengate/inference.py:36-180) and its state-span
helpers (tokengate/e2e_gate/gate_module/gate_forward.py:664-689):
  * ids carry exactly one STATE_START_ID (-1001) ... STATE_END_ID (-1002) pair
    marking the prunable document; split_state_span strips them and returns
    (clean_ids, start, end), raising ValueError on malformed spans;
  * generate runs the gated prefill on the B200 kernels and, for
    max_new_tokens > 1 (default 20, as the reference), greedy decoding over
    the gated KV cache (decode.generate_batch), returning a GenerateOutput
    with the reference's fields;
  * load_model takes a gate .pt, or a local run directory in which the
    newest-stage gate wins (swa_gate_*.pt > gate_final.pt > gate_step*.pt,
    tokengate/inference.py:38-59). Both gate kinds load: the linear
    log-sigmoid gate ({"state_dict": {"readout.weight"}, "metadata"}) and the
    finalized E2EGate with its scoring branch (the reference's save_gate
    format). A Hugging Face Hub id is rejected with an error: this build
    runs offline. LoRA adapters of the layers at and below the gate are not
    served (merged base weights only).
"""
import ctypes
import glob
import os
import re
import time
from dataclasses import dataclass
from typing import List, Optional, Sequence, Union

import numpy as np
import torch

from . import _lib
from .gate import SYNTHETIC_E2E_SEED, LinLogSigGate, load_gate, synthetic_e2e_gate
from .model import patch_model, rope_inv_freq_fp32, set_attention_backends_for_layers
from .prefill import prefill_batch_for_decode

STATE_START_ID = -1001
STATE_END_ID = -1002
_NO_PRUNING = 10_000_000


def split_state_span(ids: List[int]):
    """Strip the state sentinels: ids -> (clean_ids, start, end) (gate_forward.py:669-689)."""
    ids = list(ids)
    n_s, n_e = ids.count(STATE_START_ID), ids.count(STATE_END_ID)   # C-speed scans of long prompts
    s = ids.index(STATE_START_ID) if n_s == 1 else -1
    e = ids.index(STATE_END_ID) if n_e == 1 else -1
    if n_s != 1 or n_e != 1 or s >= e:
        starts = [i for i, t in enumerate(ids) if t == STATE_START_ID]
        ends = [i for i, t in enumerate(ids) if t == STATE_END_ID]
        raise ValueError(
            "ids carry no valid state span: expected exactly one STATE_START_ID followed by one "
            f"STATE_END_ID (produce ids with apply_chat_template(state=...)); found starts={starts} "
            f"ends={ends}")
    clean = list(ids[:s]) + list(ids[s + 1:e]) + list(ids[e + 1:])
    return clean, s, e - 1


def _split_state_span_tensor(ids, device=None):
    """split_state_span for the generate path: one conversion of the ids to an
    int64 array (a list of Python ints costs ~30 ns per id to convert; the
    sentinel scan and the cut are vectorized), the clean ids returned as a CPU
    int64 tensor. A CPU tensor of ids (pinned, for one asynchronous copy) is
    scanned through a zero-copy view and, when `device` is a CUDA device,
    copied whole and cut on that device. Same checks and error as
    split_state_span."""
    host = None
    if torch.is_tensor(ids):
        host = ids if ids.device.type == "cpu" else ids.cpu()
        a = host.numpy()
    else:
        a = np.asarray(ids, dtype=np.int64)
    if a.ndim != 1:
        raise ValueError(f"ids must be one flat sequence per prompt, got shape {a.shape}")
    a = np.ascontiguousarray(a, dtype=np.int64)
    # one pass over the ids in the library's host scan (two numpy compare +
    # flatnonzero passes cost ~0.1 ms per 32 k ids)
    fs, fe, ns, ne = (ctypes.c_int64() for _ in range(4))
    _lib.check(_lib.lib().tg_find_state_span(a.ctypes.data, a.size, STATE_START_ID, STATE_END_ID,
                                             ctypes.byref(fs), ctypes.byref(fe), ctypes.byref(ns),
                                             ctypes.byref(ne)))
    if ns.value != 1 or ne.value != 1 or fs.value >= fe.value:
        raise ValueError(
            "ids carry no valid state span: expected exactly one STATE_START_ID followed by one "
            f"STATE_END_ID (produce ids with apply_chat_template(state=...)); found "
            f"starts={np.flatnonzero(a == STATE_START_ID).tolist()} ends={np.flatnonzero(a == STATE_END_ID).tolist()}")
    s, e = fs.value, fe.value
    if host is not None and device is not None and torch.device(device).type == "cuda":
        d = ids if ids.device == torch.device(device) else host.to(device, non_blocking=True)
        d = d.to(torch.long)
        return torch.cat((d[:s], d[s + 1:e], d[e + 1:])), s, e - 1
    clean = np.concatenate((a[:s], a[s + 1:e], a[e + 1:])).astype(np.int64, copy=False)
    return torch.from_numpy(clean), s, e - 1


_THINK_RE = re.compile(r"<think>.*?</think>", re.DOTALL)
_THINK_OPEN_RE = re.compile(r"<think>.*", re.DOTALL)


def _strip_thinking(text: str) -> str:
    """Drop <think>...</think> blocks, a trailing unclosed one included, as the
    reference does with its answers (tokengate/generators.py:382-386)."""
    return _THINK_OPEN_RE.sub("", _THINK_RE.sub("", text)).strip()


def with_state_span(prefix: Sequence[int], state: Sequence[int], suffix: Sequence[int]) -> List[int]:
    """prefix + [STATE_START_ID] + state + [STATE_END_ID] + suffix."""
    return list(prefix) + [STATE_START_ID] + list(state) + [STATE_END_ID] + list(suffix)


@dataclass
class GenerateOutput:
    """Result of TokenGateModel.generate (one entry per input sequence)."""
    answers: List[str]
    n_kept: List[int]
    n_state: List[int]
    kept_pos: List[List[int]]
    prefill_s: float
    decode_s: float
    token_ids: List[List[int]]


class TokenGateModel:
    """A base model + gate behind one object; attribute access falls through to the model."""

    def __init__(self, model, gate, gate_layer: int, base_model: str):
        self.model = model
        self.gate = gate
        self.gate_layer = gate_layer
        self.base_model = base_model

    def __getattr__(self, name):
        return getattr(self.model, name)

    def prefill(self, ids_clean, starts, ends, K, prune_below_gate: bool = False):
        """The gated prefill on clean ids (no sentinels)."""
        return prefill_batch_for_decode(self.model, self.gate, ids_clean, starts, ends,
                                        self.gate_layer, K, prune_below_gate=prune_below_gate)

    def generate(self, ids: Union[List[int], List[List[int]]], tokenizer=None, *,
                 max_new_tokens: int = 20, max_kept_prefill_tokens: Optional[int] = None,
                 streamer=None) -> GenerateOutput:
        """Gated prefill + greedy decode (tokengate/inference.py:90-134).

        ids : one sequence or a batch (lists, int tensors or arrays), each with
            the state sentinels (ValueError otherwise).
        max_new_tokens : generation budget, default 20 like the reference
            (transformers' default generation length). 1 returns the
            prefill's first token only (time to first token).
        max_kept_prefill_tokens : K, the state tokens kept into the cache;
            None keeps all.
        streamer : optional put(cpu_ids (B, 1)) / end() receiver.
        """
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be positive")
        if torch.is_tensor(ids) or isinstance(ids, np.ndarray):
            ids = [ids] if ids.ndim == 1 else list(ids)
        elif len(ids) and isinstance(ids[0], (int, np.integer)):
            ids = [ids]
        dev = next(self.model.parameters()).device
        split = [_split_state_span_tensor(seq, dev) for seq in ids]
        clean = [s[0] for s in split]
        starts = [s[1] for s in split]
        ends = [s[2] for s in split]
        k = _NO_PRUNING if max_kept_prefill_tokens is None else max_kept_prefill_tokens
        if max_new_tokens > 1:
            # gated prefill + greedy decode over the gated KV cache (decode.generate_batch)
            from .decode import generate_batch
            eos = getattr(tokenizer, "eos_token_id", None) if tokenizer is not None else None
            r = generate_batch(self.model, self.gate, clean, starts, ends, self.gate_layer, k,
                               max_new_tokens, eos_token_id=eos, streamer=streamer)
            answers = []
            for toks, n in zip(r.token_ids, r.n_gen):
                answers.append(_strip_thinking(tokenizer.decode(toks[:n], skip_special_tokens=True))
                               if tokenizer is not None and n else "")
            kept_host = r.kept_pos.cpu()
            kept_pos = [kept_host[b, :n].tolist() for b, n in enumerate(r.n_kepts)]
            return GenerateOutput(answers=answers, n_kept=list(r.n_kepts),
                                  n_state=[e - s for s, e in zip(starts, ends)], kept_pos=kept_pos,
                                  prefill_s=r.prefill_s, decode_s=r.decode_s, token_ids=r.token_ids)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        first, _cache, kept, n_kepts, _kc = self.prefill(clean, starts, ends, k)
        # first tokens and kept positions come back in two asynchronous copies
        # into pinned memory and one synchronisation
        first_host = torch.empty(first.shape, dtype=first.dtype, pin_memory=True)
        kept_host = torch.empty(kept.shape, dtype=kept.dtype, pin_memory=True)
        first_host.copy_(first, non_blocking=True)
        kept_host.copy_(kept, non_blocking=True)
        torch.cuda.synchronize(dev)
        prefill_s = time.perf_counter() - t0
        tokens = [[int(t)] for t in first_host[:, 0].tolist()]
        if streamer is not None:
            streamer.put(first_host)
            streamer.end()
        answers = [tokenizer.decode(t) if tokenizer is not None else "" for t in tokens]
        kept_np = kept_host.numpy()
        kept_pos = [kept_np[b, :n].tolist() for b, n in enumerate(n_kepts)]
        return GenerateOutput(answers=answers, n_kept=list(n_kepts),
                              n_state=[e - s for s, e in zip(starts, ends)], kept_pos=kept_pos,
                              prefill_s=prefill_s, decode_s=0.0, token_ids=tokens)


# Qwen3 shapes of the benchmarked models (random-init: no checkpoints offline)
QWEN3_SHAPES = {
    "qwen3-1.7b": dict(hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                       rope_theta=1e6, vocab_size=151936, tie_word_embeddings=True,
                       max_position_embeddings=40960),
    "qwen3-8b": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                     num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                     rope_theta=1e6, vocab_size=151936, tie_word_embeddings=False,
                     max_position_embeddings=131072),
}


def qwen3_config(name_or_dict):
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
    kw = dict(QWEN3_SHAPES[name_or_dict]) if isinstance(name_or_dict, str) else dict(name_or_dict)
    cfg = Qwen3Config(**kw)
    cfg._attn_implementation = "eager"
    return cfg


def synthetic_qwen3(name_or_dict, seed: int = 0, device="cuda", dtype=torch.bfloat16):
    """Random-init Qwen3ForCausalLM of a named shape, built directly on `device`."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3ForCausalLM
    cfg = qwen3_config(name_or_dict)
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3ForCausalLM(cfg)
    model = model.to(dtype).eval()
    rope_inv_freq_fp32(model)     # the cast above also cast the rotary frequencies
    return model


def resolve_gate_path(checkpoint: str) -> str:
    """A checkpoint spec -> the gate .pt file (tokengate/inference.py:38-59).

    A path ending in .pt must be a file. A directory resolves to its
    newest-stage gate: the last (sorted) swa_gate_*.pt, else gate_final.pt,
    else the last gate_step*.pt. Anything else would be a Hub repo id, which
    needs a download: this build has no network path, so it raises
    FileNotFoundError naming the spec.
    """
    checkpoint = os.fspath(checkpoint)
    if checkpoint.endswith(".pt"):
        if not os.path.isfile(checkpoint):
            raise FileNotFoundError(f"gate checkpoint not found: {checkpoint}")
        return checkpoint
    if not os.path.isdir(checkpoint):
        raise FileNotFoundError(
            f"gate checkpoint {checkpoint!r} is neither a .pt file nor a local run directory "
            "(Hub ids need a download, which this offline build does not do: fetch the "
            "repository and pass its directory)")
    for pat in ("swa_gate_*.pt", "gate_final.pt", "gate_step*.pt"):
        hits = sorted(glob.glob(os.path.join(checkpoint, pat)))
        if hits:
            return hits[-1]
    raise FileNotFoundError(f"no gate checkpoint (gate_*.pt) in {checkpoint}")


def load_model(checkpoint: Optional[str] = None, base_model=None, gate_layer: Optional[int] = None,
               gate_attn: str = "b200", dtype=None, *, model: Optional[torch.nn.Module] = None,
               gate=None, device="cuda", seed: int = 0, trusted_checkpoint: bool = False) -> TokenGateModel:
    """Build a TokenGateModel on the B200 kernels (reference: tokengate/inference.py:141-180).

    checkpoint : a gate .pt or a run directory (resolve_gate_path: newest
        swa_gate_*.pt > gate_final.pt > gate_step*.pt). A finalized-gate checkpoint (the reference's
        save_gate format: state_dict with gate_branch.* weights and the
        finalized flags) is loaded with gate.load_gate; a linear log-sigmoid
        gate checkpoint ({"state_dict": {"readout.weight"}, "metadata"}) is
        loaded into LinLogSigGate. None when `gate` is passed (or for a
        random gate from `seed`). Read with torch's weights-only unpickler
        unless trusted_checkpoint.
    base_model : a QWEN3_SHAPES name / Qwen3Config kwargs (random init from
        `seed`), or a HF model id / path loadable by AutoModelForCausalLM;
        ignored when `model` is passed. Read from the checkpoint metadata when
        omitted, as in the reference.
    gate_layer : the gate's layer (metadata when omitted).
    gate_attn  : "b200" (or the reference's default name "fa2", same kernel).
    gate       : a gate module, or "e2e" for a synthetic finalized gate
                 (gate.synthetic_e2e_gate, seeded) on the model.
    """
    if dtype is None:
        dtype = torch.bfloat16
    if dtype != torch.bfloat16:
        raise NotImplementedError("the B200 kernels compute in bf16")
    meta = {}
    blob = None
    if checkpoint is not None:
        checkpoint = resolve_gate_path(checkpoint)
        blob = torch.load(checkpoint, map_location="cpu", weights_only=not trusted_checkpoint)
        meta = blob.get("metadata", {}) if isinstance(blob, dict) else {}
    if base_model is None:
        base_model = meta.get("base_model")
    if gate_layer is None:
        gate_layer = meta.get("gate_layer")
        if gate_layer is None:
            raise ValueError("no gate_layer: pass gate_layer= or use a checkpoint that records it")
    if model is None:
        if base_model is None:
            raise ValueError("no base_model: pass base_model= (a shape name, config kwargs or HF id)")
        if isinstance(base_model, (dict,)) or base_model in QWEN3_SHAPES:
            model = synthetic_qwen3(base_model, seed=seed, device=device, dtype=dtype)
        else:
            from transformers import AutoModelForCausalLM
            model = AutoModelForCausalLM.from_pretrained(base_model, dtype=dtype).to(device).eval()
    hidden = model.config.hidden_size
    dev = next(model.parameters()).device
    if isinstance(gate, str):
        if gate != "e2e":
            raise ValueError(f"gate={gate!r}: pass a module or 'e2e'")
        gate = synthetic_e2e_gate(model, int(gate_layer), seed=SYNTHETIC_E2E_SEED + seed, device=dev)
    if gate is None:
        state = blob.get("state_dict", blob) if isinstance(blob, dict) else None
        if state is not None and any(k.startswith("gate_branch.") for k in state):
            gate, _ = load_gate(blob)
            gate = gate.to(dev).float().eval()
        else:
            gate = LinLogSigGate(hidden, generator=torch.Generator().manual_seed(seed + 1))
            if state is not None:
                gate.load_state_dict(state)
            gate = gate.to(dev)
    patch_model(model)
    set_attention_backends_for_layers(model, gate_attn)
    name = base_model if isinstance(base_model, str) else "custom"
    return TokenGateModel(model, gate, int(gate_layer), name)
