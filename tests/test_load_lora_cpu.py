"""Load path and LoRA loader on CPU (module surgery, key matching, multipliers).

Mirrors the reference's own tests (tests/test_lora_loading.py:1-80): the
SVDQuant base term is stubbed per instance, as the reference does, so the
LoRA composition runs without a GPU."""
from __future__ import annotations

import json
import types

import pytest
import torch
from torch import nn

from krea2_svdquant_b200.linear import SVDQuantLinear
from krea2_svdquant_b200.load import load_svdquant_transformer, save_svdquant_checkpoint
from krea2_svdquant_b200.lora import ModuleIndex, addresses, load_svdquant_lora_adapters, parse_lora_keys
from krea2_svdquant_b200.quant import SVDQuantLinearState, make_synthetic_state
from krea2_svdquant_b200.replace import get_parent_module, iter_named_linears, replace_module


def _svdq_linear(in_features: int = 4, out_features: int = 3) -> SVDQuantLinear:
    state = SVDQuantLinearState(
        smooth_scale=torch.ones(in_features), qweight=torch.zeros(out_features, in_features // 2, dtype=torch.uint8),
        weight_scales=torch.ones(out_features, 1), l1=torch.zeros(out_features, 1), l2=torch.zeros(1, in_features),
        bias=None, group_size=in_features, original_shape=(out_features, in_features), qweight_packed=True,
        padded_in_features=in_features)
    return SVDQuantLinear(state, backend="b200")


class _ToyTransformer(nn.Module):
    def __init__(self):
        super().__init__()
        block = nn.Module()
        block.attn = nn.Module()
        block.attn.to_q = _svdq_linear()
        self.transformer_blocks = nn.ModuleList([block])


def _stub_base(mod: SVDQuantLinear, n_out: int) -> None:
    mod._forward_base = types.MethodType(lambda self, x: torch.zeros(x.shape[:-1] + (n_out,)), mod)


def test_lora_transformer_prefixed_keys(tmp_path):
    from safetensors.torch import save_file
    model = _ToyTransformer()
    down = torch.arange(8, dtype=torch.float32).reshape(2, 4) / 10
    up = torch.arange(6, dtype=torch.float32).reshape(3, 2) / 10
    f = tmp_path / "pytorch_lora_weights.safetensors"
    save_file({"transformer.transformer_blocks.0.attn.to_q.lora_A.weight": down,
               "transformer.transformer_blocks.0.attn.to_q.lora_B.weight": up,
               "transformer.transformer_blocks.0.attn.to_q.alpha": torch.tensor(4.0)}, str(f))
    report = load_svdquant_lora_adapters(model, tmp_path, scale=0.5)  # directory: file name inferred
    assert report["loaded"] == ["transformer_blocks.0.attn.to_q"]
    target = model.transformer_blocks[0].attn.to_q
    assert len(target.lora_adapters) == 1
    assert target.lora_adapters[0].multiplier == pytest.approx(0.5 * 4.0 / 2)
    _stub_base(target, 3)
    x = torch.randn(2, 4)
    expected = torch.nn.functional.linear(torch.nn.functional.linear(x, down), up) * (0.5 * 4.0 / 2)
    torch.testing.assert_close(target(x), expected)


def test_lora_flat_kohya_prefix(tmp_path):
    from safetensors.torch import save_file
    model = _ToyTransformer()
    f = tmp_path / "flat.safetensors"
    save_file({"lora_unet_transformer_blocks_0_attn_to_q.lora_down.weight": torch.zeros(2, 4),
               "lora_unet_transformer_blocks_0_attn_to_q.lora_up.weight": torch.zeros(3, 2)}, str(f))
    report = load_svdquant_lora_adapters(model, f)
    assert report["loaded"] == ["transformer_blocks.0.attn.to_q"]
    # no alpha: multiplier = scale * rank / rank
    assert model.transformer_blocks[0].attn.to_q.lora_adapters[0].multiplier == pytest.approx(1.0)


def test_lora_reports_incomplete_and_unmatched(tmp_path):
    from safetensors.torch import save_file
    model = _ToyTransformer()
    f = tmp_path / "mixed.safetensors"
    save_file({"transformer_blocks.0.attn.to_q.lora.down.weight": torch.zeros(2, 4),
               "transformer_blocks.0.attn.to_q.lora.up.weight": torch.zeros(3, 2),
               "transformer_blocks.0.attn.to_k.lora_A.weight": torch.zeros(2, 4),
               "transformer_blocks.0.attn.to_k.lora_B.weight": torch.zeros(3, 2),
               "transformer_blocks.0.ff.up.lora_A.weight": torch.zeros(2, 4)}, str(f))
    report = load_svdquant_lora_adapters(model, f)
    assert report["loaded"] == ["transformer_blocks.0.attn.to_q"]
    assert report["unmatched"] == ["transformer_blocks.0.attn.to_k"]
    assert report["incomplete"] == ["transformer_blocks.0.ff.up"]


def test_lora_strict_without_match_raises(tmp_path):
    from safetensors.torch import save_file
    f = tmp_path / "none.safetensors"
    save_file({"other.lora_A.weight": torch.zeros(2, 4), "other.lora_B.weight": torch.zeros(3, 2)}, str(f))
    with pytest.raises(ValueError):
        load_svdquant_lora_adapters(_ToyTransformer(), f)
    assert load_svdquant_lora_adapters(_ToyTransformer(), f, strict=False)["unmatched"] == ["other"]


def test_lora_shape_checks():
    mod = _svdq_linear()
    with pytest.raises(ValueError):
        mod.add_lora_adapter(torch.zeros(2, 5), torch.zeros(3, 2))
    with pytest.raises(ValueError):
        mod.add_lora_adapter(torch.zeros(2, 4), torch.zeros(4, 2))


def test_key_matching_helpers():
    assert addresses("base_model.model.transformer_blocks.3.ff.up", "transformer_blocks.3.ff.up")
    assert addresses("lora_unet_transformer_blocks_3_ff_up", "transformer_blocks.3.ff.up")
    assert not addresses("transformer_blocks.13.ff.up", "transformer_blocks.3.ff.up")
    entries = parse_lora_keys({"a.lora_linear_layer.down.weight": torch.zeros(1), "a.lora_linear_layer.up.weight":
                               torch.zeros(1), "a.network_alpha": torch.tensor(2.0),
                               "b.lora.down.weight": torch.zeros(1), "b.alpha": torch.zeros(2)})
    assert set(entries) == {"a", "b"}  # longest suffix wins: "b.lora.down.weight" is path "b"
    assert entries["a"].complete and entries["a"].alpha == 2.0
    assert not entries["b"].complete and entries["b"].alpha is None  # a non-scalar alpha is ignored


def test_module_index_resolves_like_a_scan():
    """The index lookup over "_"-boundary suffixes finds exactly the modules a scan of every
    module with the matching rule would find."""
    model = nn.Module()
    model.transformer_blocks = nn.ModuleList()
    for _ in range(12):
        blk = nn.Module()
        blk.attn = nn.Module()
        blk.attn.to_q = _svdq_linear()
        model.transformer_blocks.append(blk)
    idx = ModuleIndex.of(model)
    for path in ["transformer.transformer_blocks.1.attn.to_q", "lora_unet_transformer_blocks_11_attn_to_q",
                 "transformer_blocks.1.attn.to_k", "blocks.1.attn.to_q", "base_model.model.transformer_blocks.10.attn.to_q"]:
        scan = sorted(n for n in idx.modules if addresses(path, n))
        assert idx.resolve(path) == scan, path


class _DenseToy(nn.Module):
    def __init__(self, k=128, n=64):
        super().__init__()
        blk = nn.Module()
        blk.attn = nn.Module()
        blk.attn.to_q = nn.Linear(k, n)
        blk.attn.to_out = nn.ModuleList([nn.Linear(n, k)])
        blk.norm = nn.LayerNorm(k)
        self.transformer_blocks = nn.ModuleList([blk])
        self.proj_out = nn.Linear(k, k)


def test_replace_helpers():
    m = _DenseToy()
    names = [n for n, _ in iter_named_linears(m)]
    assert names == ["transformer_blocks.0.attn.to_q", "transformer_blocks.0.attn.to_out.0"]
    parent, leaf = get_parent_module(m, "transformer_blocks.0.attn.to_out.0")
    assert isinstance(parent, nn.ModuleList) and leaf == "0"
    new = nn.Identity()
    replace_module(m, "transformer_blocks.0.attn.to_out.0", new)
    assert m.transformer_blocks[0].attn.to_out[0] is new


def _states():
    _, sq = make_synthetic_state(8, 128, 64, 16, 64, seed=1, device="cpu")
    _, so = make_synthetic_state(8, 64, 128, 16, 64, seed=2, device="cpu")
    return {"transformer_blocks.0.attn.to_q": sq, "transformer_blocks.0.attn.to_out.0": so}


def test_checkpoint_round_trip(tmp_path):
    states = _states()
    save_svdquant_checkpoint(tmp_path, states)
    cfg = json.loads((tmp_path / "svdquant_config.json").read_text())
    assert set(cfg["layers"]) == set(states)
    model = _DenseToy()
    out = load_svdquant_transformer(model, tmp_path, backend="b200")
    assert out["_load_report"]["replaced"] == list(states)
    q = model.transformer_blocks[0].attn.to_q
    o = model.transformer_blocks[0].attn.to_out[0]
    assert isinstance(q, SVDQuantLinear) and isinstance(o, SVDQuantLinear)
    for mod, st in ((q, states["transformer_blocks.0.attn.to_q"]), (o, states["transformer_blocks.0.attn.to_out.0"])):
        assert torch.equal(mod.qweight, st.qweight)
        assert torch.equal(mod.weight_scales, st.weight_scales)
        assert torch.equal(mod.l1, st.l1.to(torch.bfloat16))
        assert mod.padded_in_features == st.qweight.shape[1] * 2
        assert mod.original_shape == tuple(st.original_shape)
    assert isinstance(model.transformer_blocks[0].norm, nn.LayerNorm)


def test_checkpoint_missing_tensors(tmp_path):
    from safetensors.torch import load_file, save_file
    save_svdquant_checkpoint(tmp_path, _states())
    t = load_file(str(tmp_path / "transformer_svdquant.safetensors"))
    del t["transformer_blocks__0__attn__to_q.l2"]
    save_file(t, str(tmp_path / "transformer_svdquant.safetensors"))
    with pytest.raises(KeyError):
        load_svdquant_transformer(_DenseToy(), tmp_path)
    out = load_svdquant_transformer(_DenseToy(), tmp_path, strict=False)
    assert out["_load_report"]["replaced"] == ["transformer_blocks.0.attn.to_out.0"]
    assert out["_load_report"]["missing"] == ["transformer_blocks__0__attn__to_q.l2"]


def test_reference_backend_names_rejected():
    with pytest.raises(ValueError):
        _svdq_linear().__class__(_svdq_linear().state, backend="pytorch_sim")


GOLDEN_CKPT = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "ckpt_small")


class _CkptToy(nn.Module):
    """The module tree the reference-written fixture checkpoint addresses."""

    def __init__(self):
        super().__init__()
        blk = nn.Module()
        blk.attn = nn.Module()
        blk.attn.to_q = nn.Linear(128, 96)
        blk.ff = nn.Module()
        blk.ff.down = nn.Linear(192, 128)
        self.transformer_blocks = nn.ModuleList([blk])


def test_loads_reference_written_checkpoint():
    """A checkpoint in the converter's layout, built and read back by the reference
    (tests/golden/gen_golden.py checkpoint_case), loads here unchanged."""
    from safetensors.torch import load_file
    model = _CkptToy()
    cfg = load_svdquant_transformer(model, GOLDEN_CKPT, backend="b200_w4a16")
    assert cfg["_load_report"]["replaced"] == ["transformer_blocks.0.attn.to_q", "transformer_blocks.0.ff.down"]
    t = load_file(GOLDEN_CKPT + "/transformer_svdquant.safetensors")
    q = model.transformer_blocks[0].attn.to_q
    d = model.transformer_blocks[0].ff.down
    assert torch.equal(q.qweight, t["transformer_blocks__0__attn__to_q.qweight_packed"])
    assert q.weight_scales.dtype == torch.float16 and torch.equal(q.weight_scales,
                                                                 t["transformer_blocks__0__attn__to_q.weight_scales"])
    assert q.bias is not None and d.bias is None
    assert q.original_shape == (96, 128) and d.original_shape == (128, 192)
    assert q.padded_in_features == 128 and d.padded_in_features == 192
    assert q.group_size == 64 and d.l1.shape == (128, 32)
