"""Host-side logic and the C-ABI boundary, on CPU (no GPU calls are made)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from tokengate_b200 import _lib, ops
from tokengate_b200.attn import _bias_bhs, resolve_backend
from tokengate_b200.inference import STATE_END_ID, STATE_START_ID, split_state_span, with_state_span

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    text = open(os.path.join(ROOT, "include", "tokengate_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(tg_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_header_symbol():
    lib = _lib.lib()
    declared = _header_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert sorted(_lib.EXPORTED) == declared
    assert lib.tg_abi_version() == _lib.ABI_VERSION


def _attn_args(**over):
    a = dict(q=1024, q_sb=0, q_ss=128, q_sh=128, k=2048, k_sb=0, k_ss=128, k_sh=128,
             v=4096, v_sb=0, v_ss=128, v_sh=128, bias=None, bias_sb=0, bias_sh=0,
             qs=None, qs_sb=0, qs_sh=0, out=8192, o_sb=0, o_ss=128, o_sh=128,
             lse=None, lse_sb=0, lse_sh=0, B=1, Sq=64, Sk=64, Hq=1, Hkv=1, D=128,
             scale=0.088, causal=1, stream=None)
    a.update(over)
    return list(a.values())


def test_abi_attention_validation_without_gpu():
    lib = _lib.lib()
    assert lib.tg_keybias_attn_fwd(*_attn_args(D=64)) == _lib.TG_ERR_UNSUPPORTED
    assert b"head_dim" in lib.tg_last_error()
    assert lib.tg_keybias_attn_fwd(*_attn_args(B=0)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_keybias_attn_fwd(*_attn_args(Hq=3, Hkv=2)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_keybias_attn_fwd(*_attn_args(Sk=32)) == _lib.TG_ERR_INVALID_ARGUMENT   # causal, Sq != Sk
    assert lib.tg_keybias_attn_fwd(*_attn_args(q=None)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_keybias_attn_fwd(*_attn_args(scale=0.0)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_keybias_attn_fwd(*_attn_args(out=8200)) == _lib.TG_ERR_ALIGNMENT


def _i32(*v):
    return (ctypes.c_int32 * len(v))(*v)


def test_abi_other_validation_without_gpu():
    lib = _lib.lib()
    # scorer: unsupported hidden size, misaligned rows
    st = lib.tg_gate_score(1024, 0, 100, 100, 4096, 1, _i32(0), _i32(10), 8192, 16, None)
    assert st == _lib.TG_ERR_UNSUPPORTED
    st = lib.tg_gate_score(1030, 0, 2048, 2048, 4096, 1, _i32(0), _i32(10), 8192, 16, None)
    assert st == _lib.TG_ERR_ALIGNMENT
    # top-k: k > n_state, state outside the sequence, n_kept > n_alloc, bad dtype
    args = lambda n, k, s0, L, na, dt=1: (1024, 64, 1, _i32(n), _i32(k), _i32(s0), _i32(L), na,
                                          2048, na, 4096, na, dt, None, 0, None)
    assert lib.tg_topk_select(*args(10, 11, 0, 10, 20)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_topk_select(*args(10, 0, 0, 10, 20)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_topk_select(*args(10, 5, 5, 10, 20)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_topk_select(*args(10, 5, 0, 12, 6)) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_topk_select(*args(10, 5, 0, 12, 20, dt=2)) == _lib.TG_ERR_INVALID_ARGUMENT
    # gather: tensor count, alignment, n_valid range
    g = _lib.GatherTensor(src=4096, dst=8192, src_batch_stride=0, src_row_stride=256, src_seg_stride=0,
                          dst_batch_stride=0, dst_row_stride=256, dst_seg_stride=0, seg_bytes=256,
                          n_seg=1, reserved=0)
    arr = (_lib.GatherTensor * 1)(g)
    assert lib.tg_gather_rows(arr, 0, 1024, 8, 1, 8, _i32(8), None) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_gather_rows(arr, 17, 1024, 8, 1, 8, _i32(8), None) == _lib.TG_ERR_INVALID_ARGUMENT
    bad = _lib.GatherTensor.from_buffer_copy(g)
    bad.seg_bytes = 250
    assert lib.tg_gather_rows((_lib.GatherTensor * 1)(bad), 1, 1024, 8, 1, 8, _i32(8), None) == \
        _lib.TG_ERR_ALIGNMENT
    assert lib.tg_gather_rows(arr, 1, 1024, 8, 1, 8, _i32(9), None) == _lib.TG_ERR_INVALID_ARGUMENT
    assert lib.tg_gather_rows(arr, 1, 1024, 8, 1, 0, _i32(0), None) == _lib.TG_OK   # nothing to do


def test_status_to_exception():
    with pytest.raises(_lib.TokenGateUnsupportedError):
        lib = _lib.lib()
        _lib.check(lib.tg_keybias_attn_fwd(*_attn_args(D=64)))
    with pytest.raises(ValueError):
        _lib.check(_lib.lib().tg_keybias_attn_fwd(*_attn_args(B=0)))


def test_wrappers_have_no_cpu_path():
    q = torch.zeros(1, 8, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.keybias_attention(q, q, q)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gate_score(torch.zeros(1, 8, 256, dtype=torch.bfloat16), torch.zeros(256), [0], [8])
    with pytest.raises(ValueError, match="CUDA"):
        ops.topk_select(torch.zeros(1, 8), [8], [2], [0], [8], 8)


def test_state_span():
    ids = with_state_span([1, 2], [10, 11, 12], [3])
    assert ids == [1, 2, STATE_START_ID, 10, 11, 12, STATE_END_ID, 3]
    assert split_state_span(ids) == ([1, 2, 10, 11, 12, 3], 2, 5)
    for bad in ([1, 2, 3], [STATE_END_ID, 1, STATE_START_ID], [STATE_START_ID, STATE_START_ID, 1, STATE_END_ID],
                [STATE_START_ID, 1, STATE_END_ID, STATE_END_ID]):
        with pytest.raises(ValueError):
            split_state_span(bad)


def test_find_state_span_matches_numpy():
    """The library's host scan: counts and first positions of both sentinels,
    against numpy, on random ids with 0, 1 or 2 of each (and empty input)."""
    L = _lib.lib()
    rng = np.random.default_rng(3)
    for n in (0, 1, 7, 1000, 32768):
        for _ in range(6):
            a = rng.integers(0, 151000, n).astype(np.int64)
            for sid in (STATE_START_ID, STATE_END_ID):
                for pos in rng.integers(0, max(n, 1), rng.integers(0, 3)) if n else ():
                    a[pos] = sid
            out = [ctypes.c_int64() for _ in range(4)]
            assert L.tg_find_state_span(a.ctypes.data, a.size, STATE_START_ID, STATE_END_ID,
                                        *[ctypes.byref(o) for o in out]) == 0
            fs, fe, ns, ne = (o.value for o in out)
            ss, ee = np.flatnonzero(a == STATE_START_ID), np.flatnonzero(a == STATE_END_ID)
            assert (ns, ne) == (len(ss), len(ee))
            assert fs == (ss[0] if len(ss) else -1) and fe == (ee[0] if len(ee) else -1)


def test_state_span_tensor_inputs():
    """The generate path's splitter takes a list, an int64 / int32 CPU tensor
    or a numpy array; on CPU (no CUDA device given) every form gives the
    list's clean ids and span, and invalid spans raise for tensors too."""
    from tokengate_b200.inference import _split_state_span_tensor
    ids = with_state_span([1, 2], [10, 11, 12], [3])
    want = ([1, 2, 10, 11, 12, 3], 2, 5)
    for form in (ids, torch.tensor(ids), torch.tensor(ids, dtype=torch.int32), np.asarray(ids)):
        clean, s, e = _split_state_span_tensor(form)
        assert (clean.tolist(), s, e) == want
        clean, s, e = _split_state_span_tensor(form, torch.device("cpu"))
        assert (clean.tolist(), s, e) == want
    for bad in ([1, 2, 3], [STATE_END_ID, 1, STATE_START_ID]):
        with pytest.raises(ValueError):
            _split_state_span_tensor(torch.tensor(bad))


def test_bias_layouts():
    B, H, S = 2, 4, 5
    s = torch.arange(S, dtype=torch.bfloat16)
    bs = torch.arange(B * S, dtype=torch.float32).view(B, S)
    sh = torch.arange(S * H, dtype=torch.float32).view(S, H)
    bsh = torch.arange(B * S * H, dtype=torch.float32).view(B, S, H)
    full = lambda t: torch.broadcast_to(t, (B, H, S))
    assert torch.equal(full(_bias_bhs(s, False, B, H, S)), s.float().view(1, 1, S).expand(B, H, S))
    assert torch.equal(full(_bias_bhs(bs, False, B, H, S)), bs.view(B, 1, S).expand(B, H, S))
    assert torch.equal(full(_bias_bhs(sh, True, B, H, S)), sh.t().view(1, H, S).expand(B, H, S))
    assert torch.equal(full(_bias_bhs(bsh, True, B, H, S)), bsh.permute(0, 2, 1))
    for b in (_bias_bhs(s, False, B, H, S), _bias_bhs(sh, True, B, H, S), _bias_bhs(bsh, True, B, H, S)):
        assert b.dtype == torch.float32 and b.stride(-1) == 1
    with pytest.raises(ValueError):
        _bias_bhs(torch.zeros(S + 1), False, B, H, S)


def test_backend_names():
    assert resolve_backend("b200", causal=True) == "b200"
    assert resolve_backend("fa2-bias", causal=False) == "b200"
    for bad in ("flex", "sdpa", "cudnn", "aug-fa4"):
        with pytest.raises(ValueError):
            resolve_backend(bad, causal=False)


def test_resolve_gate_path_run_directory(tmp_path):
    """A run directory resolves to its newest-stage gate (tokengate/inference.py:38-59):
    swa_gate_* > gate_final > gate_step*, the last of each sorted; a .pt path
    must exist; a spec that is neither (a Hub id) is an error offline."""
    from tokengate_b200.inference import resolve_gate_path
    d = tmp_path / "run"
    d.mkdir()
    with pytest.raises(FileNotFoundError):
        resolve_gate_path(str(d))                      # no gate in it yet
    for n in ("gate_step100.pt", "gate_step200.pt"):
        (d / n).write_bytes(b"x")
    assert resolve_gate_path(str(d)) == str(d / "gate_step200.pt")
    (d / "gate_final.pt").write_bytes(b"x")
    assert resolve_gate_path(str(d)) == str(d / "gate_final.pt")
    for n in ("swa_gate_a.pt", "swa_gate_b.pt"):
        (d / n).write_bytes(b"x")
    assert resolve_gate_path(d) == str(d / "swa_gate_b.pt")
    assert resolve_gate_path(str(d / "gate_final.pt")) == str(d / "gate_final.pt")
    with pytest.raises(FileNotFoundError):
        resolve_gate_path(str(d / "missing.pt"))
    with pytest.raises(FileNotFoundError, match="offline"):
        resolve_gate_path("liana313/tokengate-some-repo")


def test_load_model_from_run_directory_cpu(tmp_path):
    """load_model(run_dir) loads the directory's newest linear gate and its metadata."""
    from tokengate_b200.inference import load_model
    small = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
                 num_key_value_heads=1, head_dim=128, vocab_size=300, rope_theta=1e6)
    d = tmp_path / "run"
    d.mkdir()
    for name, fill in (("gate_step10.pt", 1.0), ("gate_final.pt", 2.0)):
        torch.save({"state_dict": {"readout.weight": torch.full((1, 256), fill)},
                    "metadata": {"gate_layer": 1}}, d / name)
    tm = load_model(str(d), base_model=small, device="cpu")
    assert tm.gate_layer == 1
    assert torch.equal(tm.gate.readout.weight.detach(), torch.full((1, 256), 2.0))


def test_rotary_frequencies_stay_fp32():
    """A model cast to bf16 after construction gets float32 rotary frequencies
    back (patch_model / synthetic_qwen3): the rotary cos at position 30000
    then matches the float64 angle to bf16 rounding, as a from_pretrained(bf16)
    model does; with bf16 frequencies it is off by whole turns."""
    from tokengate_b200.inference import qwen3_config
    from tokengate_b200.model import patch_model
    from transformers.models.qwen3.modeling_qwen3 import Qwen3ForCausalLM
    small = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
                 num_key_value_heads=1, head_dim=128, vocab_size=300, rope_theta=1e6)
    m = Qwen3ForCausalLM(qwen3_config(small)).to(torch.bfloat16)
    pos = torch.tensor([[0, 1000, 8000, 30000]])
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float64) / 128))
    ang = pos[0, :, None].double() * inv
    x = torch.zeros(1, 4, 256, dtype=torch.bfloat16)
    c_bad, _ = m.model.rotary_emb(x, pos)
    assert (c_bad[0, :, :64].double() - ang.cos()).abs().max() > 0.5
    patch_model(m)
    assert m.model.rotary_emb.inv_freq.dtype == torch.float32
    c, s = m.model.rotary_emb(x, pos)
    assert (c[0, :, :64].double() - ang.cos()).abs().max() < 1.5e-2
    assert (s[0, :, :64].double() - ang.sin()).abs().max() < 1.5e-2
