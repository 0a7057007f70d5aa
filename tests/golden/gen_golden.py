"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference project is importable (its ``src``
directory on ``sys.path``: ``--ref`` or the ``KREA2_REF_SRC`` environment variable).  The script
imports the reference's own functions and records their inputs and outputs:

* ``quantize_symmetric_int4`` / ``pack_int4`` / ``unpack_int4``
  (src/krea2_svdquant/quant/pack.py:6-70);
* ``svd_lowrank`` / ``compute_smooth_scale`` (src/krea2_svdquant/quant/svd.py:26-86);
* ``svdquant_linear_sim`` in bf16 and float32 (svd.py:119-163);
* ``SVDQuantLinear(backend="pytorch_sim")`` with a LoRA adapter
  (src/krea2_svdquant/runtime/linear.py:62-161).

Tensors are stored in ``.npz`` files next to this script; bf16 tensors are
stored as their uint16 bit patterns (keys ending in ``__bf16``).

    python tests/golden/gen_golden.py --ref <reference checkout>/src
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t: torch.Tensor, key: str, out: dict) -> None:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        out[key + "__bf16"] = t.view(torch.int16).numpy().view(np.uint16)
    elif t.dtype == torch.float16:
        out[key + "__fp16"] = t.numpy()
    else:
        out[key] = t.numpy()


def baseline_inputs(m, k, n, rank, group, *, seed, bias=True, scale_dtype=torch.bfloat16,
                    clamp_smooth=False, ref=None):
    """The BASELINE.json synthetic recipe at a small size, built with the reference's functions."""
    svd_lowrank = ref["svd_lowrank"]
    q4 = ref["quantize_symmetric_int4"]
    pack = ref["pack_int4"]
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    outl = torch.randperm(k, generator=g)[: max(1, k // 100)]
    x[:, outl] *= 20
    x = x.bfloat16()
    w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    if clamp_smooth:
        s = ref["compute_smooth_scale"](x.float().abs().amax(0), w)
    else:
        s = (x.float().abs().amax(0).sqrt() / w.float().abs().amax(0).clamp_min(1e-8).sqrt()).bfloat16()
    mig = w * s.unsqueeze(0)
    l1, l2 = svd_lowrank(mig, rank)
    res = mig.float() - l1.float() @ l2.float()
    q, ws = q4(res, group_size=group, dim=1)
    b = (torch.randn(n, generator=g) * 0.01).bfloat16() if bias else None
    return dict(x=x, smooth=s, qweight=pack(q), weight_scales=ws.to(scale_dtype), l1=l1, l2=l2, bias=b)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("KREA2_REF_SRC"), required="KREA2_REF_SRC" not in os.environ,
                    help="the reference checkout's src directory (or set KREA2_REF_SRC)")
    ap.add_argument("--only", default=None, help="write only this fixture (file stem)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from krea2_svdquant.quant.pack import pack_int4, quantize_symmetric_int4, unpack_int4
    from krea2_svdquant.quant.svd import (SVDQuantLinearState, compute_smooth_scale, svd_lowrank,
                                          svdquant_linear_sim)
    from krea2_svdquant.runtime.linear import SVDQuantLinear

    ref = dict(svd_lowrank=svd_lowrank, quantize_symmetric_int4=quantize_symmetric_int4,
               pack_int4=pack_int4, compute_smooth_scale=compute_smooth_scale)
    torch.manual_seed(0)

    def linear_case(name, m, k, n, rank, group, *, seed, scale_dtype=torch.bfloat16, bias=True,
                    clamp_smooth=False, lora=None):
        inp = baseline_inputs(m, k, n, rank, group, seed=seed, bias=bias, scale_dtype=scale_dtype,
                              clamp_smooth=clamp_smooth, ref=ref)
        k_pad = inp["qweight"].shape[1] * 2
        st = SVDQuantLinearState(inp["smooth"], inp["qweight"], inp["weight_scales"], inp["l1"],
                                 inp["l2"], inp["bias"], group, (n, k), True, k_pad)
        out: dict = {"group": np.int64(group), "k_in": np.int64(k), "k_pad": np.int64(k_pad)}
        for key, t in inp.items():
            if t is not None:
                _np(t, key, out)
        x = inp["x"]
        x_hat = x / inp["smooth"]
        _np(x_hat, "x_hat", out)
        for ag in (64, 128):
            qa, sa = quantize_symmetric_int4(x_hat, group_size=ag, dim=1)
            out[f"act_q_g{ag}"] = qa.numpy()
            _np(sa, f"act_scale_g{ag}", out)
            out[f"act_packed_g{ag}"] = pack_int4(qa).numpy()
            assert torch.equal(unpack_int4(pack_int4(qa), qa.shape[-1]), qa)
        _np(torch.nn.functional.linear(x_hat, inp["l2"]), "mid_ref", out)
        _np(svdquant_linear_sim(x, st), "y_sim_bf16", out)
        _np(svdquant_linear_sim(x.float(), st), "y_sim_fp32", out)
        if lora is not None:
            rl, scale, alpha = lora
            g = torch.Generator().manual_seed(seed + 1)
            down = (torch.randn(rl, k, generator=g) * 0.01).bfloat16()
            up = (torch.randn(n, rl, generator=g) * 0.01).bfloat16()
            mod = SVDQuantLinear(st, backend="pytorch_sim")
            mod.add_lora_adapter(down, up, scale=scale, network_alpha=alpha)
            _np(down, "lora_down", out)
            _np(up, "lora_up", out)
            out["lora_mult"] = np.float64(mod.lora_adapters[0].multiplier)
            with torch.no_grad():
                _np(mod(x), "y_mod_bf16", out)
                _np(mod(x.float()), "y_mod_fp32", out)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print("wrote", name, {k2: v.shape for k2, v in out.items()})

    if args.only == "weight_quant_fp32":
        weight_quant_case(quantize_symmetric_int4, pack_int4)
        return
    if args.only == "ckpt_small":
        checkpoint_case()
        return
    # BASELINE recipe (config-1 distributions) at a fixture-friendly size.
    linear_case("linear_g64", 64, 1024, 256, 32, 64, seed=1, lora=(16, 0.8, 8.0))
    # K not a group multiple: padded to 192 inside quantize_symmetric_int4 (pack.py:12-16).
    linear_case("linear_pad", 16, 130, 64, 8, 64, seed=2)
    # Converter format: group 128, fp16 weight scales, mlp rank 64, no bias (convert_simulated.py:201-208).
    linear_case("linear_g128_fp16", 32, 512, 128, 64, 128, seed=3, scale_dtype=torch.float16, bias=False)
    # Reference smoothing clamp to [0.25, 4] (svd.py:26-30).
    linear_case("linear_clamped", 32, 256, 64, 16, 64, seed=4, clamp_smooth=True)

    # Quantizer edge cases on bf16 inputs: exact half ties, zero and tiny groups, +/-8 clamp.
    rows = []
    r = torch.zeros(64)
    r[:16] = torch.tensor([7.0, 0.5, 1.5, 2.5, 3.5, -0.5, -1.5, -2.5, -3.5, 4.5, -4.5, 5.5, -5.5, 6.5, -6.5, -7.0])
    rows.append(r)
    rows.append(torch.zeros(64))                       # all-zero group -> scale bf16(1e-8)/7
    rows.append(torch.full((64,), 1e-30))              # tiny group below the clamp
    r = torch.linspace(-3.0, 3.0, 64)
    r[5] = -3.25                                       # most negative dominates -> q = -7 / -8 path
    rows.append(r)
    gen = torch.Generator().manual_seed(5)
    rows.append(torch.randn(64, generator=gen) * 1e3)
    rows.append(torch.randn(64, generator=gen) * 1e-3)
    xe = torch.stack(rows).bfloat16()
    qe, se = quantize_symmetric_int4(xe, group_size=64, dim=1)
    out = {}
    _np(xe, "x", out)
    out["q"] = qe.numpy()
    _np(se, "scales", out)
    out["packed"] = pack_int4(qe).numpy()
    qf, sf = quantize_symmetric_int4(xe.float(), group_size=32, dim=1)
    out["q_fp32_g32"] = qf.numpy()
    out["scales_fp32_g32"] = sf.numpy()
    np.savez_compressed(os.path.join(HERE, "quant_edges.npz"), **out)
    print("wrote quant_edges")
    weight_quant_case(quantize_symmetric_int4, pack_int4)
    checkpoint_case()


def checkpoint_case() -> None:
    """A two-layer transformer-only checkpoint in the converter's on-disk layout
    (scripts/convert_simulated.py:136-221): per layer the reference's smoothing, low-rank
    factors and INT4 residual (fp16 scales), saved with safetensors plus svdquant_config.json.
    The reference's own loader (runtime/load.py:52-132) reads it back into a toy transformer
    and its pytorch_sim modules give the recorded fp32 outputs."""
    import json
    import shutil

    from safetensors.torch import save_file
    from torch import nn

    from krea2_svdquant.quant.pack import pack_int4, quantize_symmetric_int4
    from krea2_svdquant.quant.svd import compute_smooth_scale, svd_lowrank
    from krea2_svdquant.runtime.linear import SVDQuantLinear
    from krea2_svdquant.runtime.load import load_svdquant_transformer

    out_dir = os.path.join(HERE, "ckpt_small")
    shutil.rmtree(out_dir, ignore_errors=True)
    os.makedirs(out_dir)
    g = torch.Generator().manual_seed(21)
    layers = {"transformer_blocks.0.attn.to_q": (96, 128, 16, True), "transformer_blocks.0.ff.down": (128, 192, 32, False)}
    tensors, meta = {}, {"base_model": "krea/Krea-2-Turbo", "format": "krea2-svdquant-transformer-v1",
                         "target_component": "transformer", "weight_bits": 4, "activation_bits": 16,
                         "group_size": 64, "layers": {}}
    inputs = {}
    for name, (n, k, rank, bias) in layers.items():
        w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
        x = torch.randn(24, k, generator=g)
        x[:, ::17] *= 10.0
        smooth = compute_smooth_scale(x.abs().amax(0), w, 0.25, 4.0).cpu()
        mig = w * smooth.unsqueeze(0)
        l1, l2 = svd_lowrank(mig, rank)
        res = mig.float() - l1.float() @ l2.float()
        q, sc = quantize_symmetric_int4(res, group_size=64, dim=1)
        key = name.replace(".", "__")
        tensors[f"{key}.qweight_packed"] = pack_int4(q)
        tensors[f"{key}.weight_scales"] = sc.to(torch.float16)
        tensors[f"{key}.smooth_scale"] = smooth.to(torch.bfloat16)
        tensors[f"{key}.l1"] = l1.to(torch.bfloat16)
        tensors[f"{key}.l2"] = l2.to(torch.bfloat16)
        if bias:
            tensors[f"{key}.bias"] = (torch.randn(n, generator=g) * 0.01).bfloat16()
        meta["layers"][name] = {"rank": rank, "group_size": 64, "shape": [n, k], "calibrated": True}
        inputs[name] = x.bfloat16()
    save_file(tensors, os.path.join(out_dir, "transformer_svdquant.safetensors"))
    with open(os.path.join(out_dir, "svdquant_config.json"), "w") as f:
        json.dump(meta, f, indent=2)

    class Toy(nn.Module):
        def __init__(self):
            super().__init__()
            blk = nn.Module()
            blk.attn = nn.Module()
            blk.attn.to_q = nn.Linear(128, 96)
            blk.ff = nn.Module()
            blk.ff.down = nn.Linear(192, 128)
            self.transformer_blocks = nn.ModuleList([blk])

    toy = Toy()
    report = load_svdquant_transformer(toy, out_dir, backend="pytorch_sim")
    assert report["_load_report"]["replaced"] == list(layers)
    outs = {}
    for name in layers:
        mod = toy.get_submodule(name)
        assert isinstance(mod, SVDQuantLinear)
        with torch.no_grad():
            outs[name.replace(".", "__") + "__x"] = inputs[name].float().numpy()
            outs[name.replace(".", "__") + "__y_fp32"] = mod(inputs[name].float()).numpy()
    np.savez_compressed(os.path.join(out_dir, "reference_outputs.npz"), **outs)
    print("wrote ckpt_small")


def weight_quant_case(quantize_symmetric_int4, pack_int4) -> None:
    """The converter's weight quantization (convert_simulated.py:197-203): an fp32 residual
    quantized along K with fp32 scales, then packed; K = 200 is not a group multiple."""
    g = torch.Generator().manual_seed(9)
    w = torch.randn(48, 200, generator=g) * 0.02
    w[:, ::37] *= 15.0                                   # outlier columns
    w[3] = 0.0                                           # all-zero row -> 1e-8 clamp
    w[4, :64] = torch.arange(64, dtype=torch.float32) % 15 - 7.0  # amax 7: scale exactly 1
    w[4, 1:14] = torch.tensor([0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.5, -0.5, -1.5, -2.5, -3.5, -4.5, -5.5])  # ties
    w[5, :64] = -w[5, :64].abs()                         # negative maximum
    w[6] = w[6] * 1e-6
    out = {"w": w.numpy()}
    for group in (64, 128):
        q, sc = quantize_symmetric_int4(w, group_size=group, dim=1)
        out[f"q_g{group}"] = q.numpy()
        out[f"packed_g{group}"] = pack_int4(q).numpy()
        out[f"scales_g{group}"] = sc.numpy()
        out[f"scales_fp16_g{group}"] = sc.to(torch.float16).numpy()
    np.savez_compressed(os.path.join(HERE, "weight_quant_fp32.npz"), **out)
    print("wrote weight_quant_fp32")


if __name__ == "__main__":
    main()
