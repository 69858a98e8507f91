"""MLX safetensors checkpoint loading (host logic, CPU tensors).

A small checkpoint in the MLX quantized layout is written here byte by byte
(safetensors container: 8-byte header length, JSON header, raw data) with two
shards and an index, a default quantization of bits 4 / group 64, one module
overridden to 8 bits and one left unquantized; the loader must return the
same arrays, honour the per-module specs, and fuse projections.
"""

from __future__ import annotations

import json
import struct

import numpy as np
import pytest
import torch

import __graft_entry__
from oracle import bf16 as obf16
from oracle import qmm as oqmm


@pytest.fixture(scope="module")
def pkg():
    return __graft_entry__.load_package()


def _write_safetensors(path, tensors):
    """tensors: name -> (dtype tag, numpy array of the storage dtype)."""
    header, blobs, off = {}, [], 0
    for name, (tag, arr) in tensors.items():
        raw = np.ascontiguousarray(arr).astype(arr.dtype.newbyteorder("<")).tobytes()
        header[name] = {"dtype": tag, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "mlx"}
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _linear(rng, n, k, bits=4):
    if bits == 4:
        w, s, b = oqmm.synth_weights(rng, n, k)
    else:
        w = rng.integers(0, 2**32, size=(n, k * bits // 32), dtype=np.uint64).astype(np.uint32)
        s = obf16.from_f32(rng.random((n, k // 64), dtype=np.float32))
        b = obf16.from_f32(rng.random((n, k // 64), dtype=np.float32))
    return w, s, b


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("mlx_ckpt")
    rng = np.random.default_rng(5)
    h, inter = 128, 256
    arrays = {}
    shard = {}
    for layer in range(2):
        pre = f"model.layers.{layer}"
        for name, n, k in (("self_attn.q_proj", 128, h), ("self_attn.k_proj", 64, h),
                           ("self_attn.v_proj", 64, h), ("self_attn.o_proj", h, 128),
                           ("mlp.gate_proj", inter, h), ("mlp.up_proj", inter, h),
                           ("mlp.down_proj", h, inter)):
            bits = 8 if (layer == 1 and name == "mlp.down_proj") else 4
            w, s, b = _linear(rng, n, k, bits)
            p = f"{pre}.{name}"
            arrays[p] = (w, s, b, bits)
            f = f"model-0000{layer + 1}-of-00002.safetensors"
            shard[f"{p}.weight"] = (f, ("U32", w))
            shard[f"{p}.scales"] = (f, ("BF16", s))
            shard[f"{p}.biases"] = (f, ("BF16", b))
    emb = obf16.from_f32(rng.standard_normal((32, h)).astype(np.float32))
    shard["model.embed_tokens.weight"] = ("model-00001-of-00002.safetensors", ("BF16", emb))
    files = {}
    for name, (f, t) in shard.items():
        files.setdefault(f, {})[name] = t
    for f, t in files.items():
        _write_safetensors(d / f, t)
    (d / "model.safetensors.index.json").write_text(json.dumps(
        {"metadata": {}, "weight_map": {k: v[0] for k, v in shard.items()}}))
    (d / "config.json").write_text(json.dumps({
        "model_type": "test", "quantization": {
            "group_size": 64, "bits": 4,
            "model.layers.1.mlp.down_proj": {"group_size": 64, "bits": 8},
            "model.embed_tokens": False}}))
    return d, arrays


def _bits16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_loader_returns_the_stored_arrays(pkg, ckpt):
    d, arrays = ckpt
    mods = pkg.checkpoint.load_quantized_linears(d, "cpu")
    assert sorted(mods) == sorted(arrays)
    for p, (w, s, b, bits) in arrays.items():
        m = mods[p]
        assert m.bits == bits and m.group_size == 64 and m.mode == "affine"
        assert np.array_equal(m.weight.numpy().view(np.uint32), w)
        assert np.array_equal(_bits16(m.scales), s) and np.array_equal(_bits16(m.biases), b)
        assert m.scales.dtype == torch.bfloat16


def test_per_module_spec_and_eligibility(pkg, ckpt):
    d, _ = ckpt
    ck = pkg.checkpoint.Checkpoint(d)
    assert ck.quant_spec("model.layers.1.mlp.down_proj")["bits"] == 8
    assert ck.quant_spec("model.embed_tokens") is None
    assert "model.embed_tokens" not in ck.quantized_linear_paths()
    mods = pkg.checkpoint.load_quantized_linears(d, "cpu")
    assert not pkg.is_verify_eligible(mods["model.layers.1.mlp.down_proj"])
    assert pkg.is_verify_eligible(mods["model.layers.0.mlp.down_proj"], path="model.layers.0.mlp.down_proj")


def test_predicate_filters_modules(pkg, ckpt):
    d, _ = ckpt
    mods = pkg.checkpoint.load_quantized_linears(d, "cpu", predicate=lambda p: p.endswith("o_proj"))
    assert sorted(mods) == ["model.layers.0.self_attn.o_proj", "model.layers.1.self_attn.o_proj"]


def test_fused_layouts(pkg, ckpt):
    d, arrays = ckpt
    mods = pkg.checkpoint.load_quantized_linears(d, "cpu")
    pre = "model.layers.0"
    qkv = pkg.checkpoint.fuse_rows([mods[f"{pre}.self_attn.{n}_proj"] for n in "qkv"])
    want = np.concatenate([arrays[f"{pre}.self_attn.{n}_proj"][0] for n in "qkv"])
    assert np.array_equal(qkv.q.numpy().view(np.uint32), want)
    gu = pkg.checkpoint.fuse_gate_up(mods[f"{pre}.mlp.gate_proj"], mods[f"{pre}.mlp.up_proj"])
    g, u = arrays[f"{pre}.mlp.gate_proj"][0], arrays[f"{pre}.mlp.up_proj"][0]
    inter = g.shape[0]
    want = np.stack([g.reshape(inter // 16, 16, -1), u.reshape(inter // 16, 16, -1)], 1).reshape(2 * inter, -1)
    assert np.array_equal(gu.q.numpy().view(np.uint32), want)
    with pytest.raises(NotImplementedError):
        pkg.checkpoint.fuse_rows([mods[f"{pre}.mlp.down_proj"], mods["model.layers.1.mlp.down_proj"]])


def test_rejects_non_safetensors(pkg, tmp_path):
    (tmp_path / "x.safetensors").write_bytes(b"\x01")
    with pytest.raises(ValueError):
        pkg.checkpoint.Checkpoint(tmp_path)


def test_single_file_quantization_config_and_bias(pkg, tmp_path):
    """One safetensors file without an index, the quantization under
    ``quantization_config``, a projection with an additive ``.bias``, and a
    projection stored without ``.biases`` (not affine int4: refused)."""
    rng = np.random.default_rng(11)
    w, s, b = _linear(rng, 64, 128)
    bias = obf16.from_f32(rng.standard_normal(64).astype(np.float32))
    w2, s2, _ = _linear(rng, 64, 128)
    _write_safetensors(tmp_path / "model.safetensors", {
        "proj.weight": ("U32", w), "proj.scales": ("BF16", s), "proj.biases": ("BF16", b),
        "proj.bias": ("BF16", bias)})
    (tmp_path / "config.json").write_text(json.dumps({"quantization_config": {"group_size": 64, "bits": 4}}))
    mods = pkg.checkpoint.load_quantized_linears(tmp_path, "cpu")
    assert sorted(mods) == ["proj"]
    m = mods["proj"]
    assert (m.in_features, m.out_features) == (128, 64)
    assert np.array_equal(_bits16(m.bias), bias)
    with pytest.raises(NotImplementedError):
        pkg.checkpoint.fuse_rows([m])

    other = tmp_path / "no_biases"
    other.mkdir()
    _write_safetensors(other / "model.safetensors", {"p.weight": ("U32", w2), "p.scales": ("BF16", s2)})
    (other / "config.json").write_text(json.dumps({"quantization": {"group_size": 64, "bits": 4,
                                                                    "mode": "mxfp4"}}))
    with pytest.raises(NotImplementedError):
        pkg.checkpoint.load_quantized_linears(other, "cpu")


def test_rejects_tensor_size_mismatch(pkg, tmp_path):
    """A header whose data offsets disagree with the shape is refused."""
    rng = np.random.default_rng(12)
    w, s, b = _linear(rng, 64, 128)
    _write_safetensors(tmp_path / "model.safetensors", {"p.weight": ("U32", w), "p.scales": ("BF16", s),
                                                        "p.biases": ("BF16", b)})
    ck = pkg.checkpoint.Checkpoint(tmp_path)
    ref = ck.tensors["p.weight"]
    bad = pkg.checkpoint.TensorRef(ref.file, ref.dtype, (64, 8), ref.begin, ref.end)
    with pytest.raises(ValueError):
        bad.numpy()


@pytest.mark.gpu
def test_loaded_layers_run_on_the_gpu(pkg, ckpt):
    """Loaded to the GPU: a verify linear of the checkpoint matches the oracle
    on the stored arrays, and the fused gate|up + SiLU launch built from the
    checkpoint equals SiLU*up of the two loaded projections."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dflash_mlx_b200.moe import silu_mul

    d, arrays = ckpt
    dev = torch.device("cuda:0")
    mods = pkg.checkpoint.load_quantized_linears(d, dev)
    rng = np.random.default_rng(9)
    x = oqmm.synth_x(rng, 16, 128)
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    p = "model.layers.0.self_attn.q_proj"
    w, s, b, _ = arrays[p]
    y = pkg.VerifyQuantizedLinear.from_quantized(mods[p])(xd)
    ref = obf16.to_f32(oqmm.qmm(x, w, s, b)).astype(np.float64)
    got = y.float().cpu().numpy().astype(np.float64)
    assert not (np.abs(got - ref) > 1e-2 + 2e-2 * np.abs(ref)).any()
    pre = "model.layers.1.mlp"
    gu = pkg.checkpoint.pair_pack(pkg.checkpoint.fuse_gate_up(mods[f"{pre}.gate_proj"], mods[f"{pre}.up_proj"]))
    h = pkg.gate_up_silu(xd, gu.q, gu.s, gu.b)
    gate = pkg.qmm_w4g64(xd, mods[f"{pre}.gate_proj"].weight, mods[f"{pre}.gate_proj"].scales,
                         mods[f"{pre}.gate_proj"].biases)
    up = pkg.qmm_w4g64(xd, mods[f"{pre}.up_proj"].weight, mods[f"{pre}.up_proj"].scales,
                       mods[f"{pre}.up_proj"].biases)
    ref_h = silu_mul(gate, up).float().cpu().numpy().astype(np.float64)
    got_h = h.float().cpu().numpy().astype(np.float64)
    assert not (np.abs(got_h - ref_h) > 1e-2 + 2e-2 * np.abs(ref_h)).any()
