"""Output writers on CPU: the dense safetensors file of SafetensorsWriter.cs and the
compressed-tensors ``pack-quantized`` checkpoint, checked against the safetensors and
compressed-tensors libraries when they are installed (results from the oracle stand in for
the kernels' outputs, which have the same layout and are bit-exact with it)."""

import json
import os

import numpy as np
import pytest
import torch

from llmcompressorsharp_b200.output import (CompressedTensorsWriter, SafetensorsWriter, load_safetensors, pack_int32,
                                            save_safetensors, signed_codes)
from llmcompressorsharp_b200.session import CompressionState
from oracle import fakequant as o_fq
from oracle import rtn as o_rtn


def test_safetensors_round_trip(tmp_path):
    g = torch.Generator().manual_seed(1)
    ts = {"a.weight": torch.randn(5, 7, generator=g), "b": torch.randn(3, generator=g).to(torch.bfloat16),
          "c": torch.randint(-100, 100, (4, 4), generator=g, dtype=torch.int32), "d": torch.zeros(0, 3),
          "e": torch.tensor([1, 2, 3], dtype=torch.int64), "f": torch.randint(0, 255, (9,), generator=g).to(torch.uint8)}
    p = str(tmp_path / "x.safetensors")
    save_safetensors(ts, p, metadata={"format": "pt"})
    back = load_safetensors(p)
    assert sorted(back) == sorted(ts)
    for k in ts:
        assert back[k].dtype == ts[k].dtype and torch.equal(back[k], ts[k]), k
    st = pytest.importorskip("safetensors.torch")
    lib = st.load_file(p)
    for k in ts:
        assert torch.equal(lib[k], ts[k]), k


def test_safetensors_writer_mirrors_reference(tmp_path):  # SafetensorsWriterTests.cs (all three cases)
    from llmcompressorsharp_b200.errors import ArgumentError

    kat = CompressionState({"a.weight": torch.tensor([-1.0, 0.0, 1.0, 2.0]), "b.weight": torch.tensor([[1.0, 2.0], [3.0, 4.0]])})
    pk = str(tmp_path / "kat.safetensors")
    SafetensorsWriter.save(kat, pk)
    assert os.path.getsize(pk) > 0
    back = SafetensorsWriter.load(pk)
    assert back["a.weight"].tolist() == [-1.0, 0.0, 1.0, 2.0] and list(back["a.weight"].shape) == [4]
    assert list(back["b.weight"].shape) == [2, 2]
    state = CompressionState({"model.layers.0.mlp.down_proj.weight": torch.ones(2, 3)})
    p = str(tmp_path / "m.safetensors")
    SafetensorsWriter.save(state, p)
    assert torch.equal(SafetensorsWriter.load(p)["model.layers.0.mlp.down_proj.weight"], torch.ones(2, 3))
    with pytest.raises(ArgumentError):
        SafetensorsWriter.save(None, p)
    with pytest.raises(ArgumentError):
        SafetensorsWriter.save(state, " ")
    with pytest.raises(FileNotFoundError):
        SafetensorsWriter.load(str(tmp_path / "missing.safetensors"))


def test_pack_int32_layout():
    v = np.array([[1, 2, -8, 7, 0, -1, 3, -3, 5]], dtype=np.int8)
    w = pack_int32(v, 4)
    assert w.shape == (1, 2) and w.dtype == np.int32
    u = (v.astype(np.int64) + 8)
    word0 = sum(int(u[0, i]) << (4 * i) for i in range(8))
    assert int(w[0, 0]) & 0xFFFFFFFF == word0
    assert int(w[0, 1]) == int(u[0, 8])  # padding zeros above
    w8 = pack_int32(np.array([[1, 2], [3, 4], [5, 6], [7, 8], [9, 10]], dtype=np.int8), 8, packed_dim=0)
    assert w8.shape == (2, 2)
    assert int(w8[0, 0]) & 0xFFFFFFFF == (129 | 131 << 8 | 133 << 16 | 135 << 24)


def _rtn_entry(w, bits, sym, strategy, gs):
    deq, q, rs, rz = o_rtn.rtn_quantize(w, o_rtn.RtnConfig(bits, sym, strategy, group_size=gs))
    m, n = w.shape
    zp = torch.from_numpy(np.asarray(rz))
    if bits <= 4:
        zp_e = zp[:, torch.arange(n) // gs] if strategy == "group" else zp.reshape(-1, 1).expand(m, n)
        codes = o_fq.pack_int4_rows(q, zp_e)
    else:
        codes = q.to(torch.uint8)
    shp = (m, -1) if strategy == "group" else (m,)
    entry = {"codes": codes, "scales": torch.from_numpy(np.asarray(rs, np.float32)).reshape(shp),
             "zero_points": zp.to(torch.int32).reshape(shp), "num_bits": bits, "symmetric": sym, "strategy": strategy,
             "group_size": gs}
    return entry, q, deq


@pytest.mark.parametrize("bits,sym,strategy", [(4, False, "group"), (4, True, "group"), (4, False, "channel"),
                                               (8, False, "group"), (8, True, "channel")])
def test_signed_codes_recover_the_codes(bits, sym, strategy):
    w = (torch.randn(24, 256, generator=torch.Generator().manual_seed(bits + 3 * sym)) * 0.02)
    entry, q, _ = _rtn_entry(w, bits, sym, strategy, 128)
    qs, zs = signed_codes(entry["codes"], entry["zero_points"], bits, sym, 256, strategy, 128)
    half = 1 << (bits - 1)
    assert np.array_equal(qs.astype(np.int64), q.numpy().astype(np.int64) - (0 if sym else half))
    zp = entry["zero_points"].numpy().astype(np.int64)
    assert np.array_equal(zs.astype(np.int64), np.zeros_like(zp) if sym else zp - half)
    assert qs.min() >= -half and qs.max() <= half - 1


@pytest.mark.parametrize("bits,sym,strategy", [(4, False, "group"), (4, True, "group"), (4, False, "channel"),
                                               (8, False, "group"), (8, True, "channel")])
def test_compressed_tensors_checkpoint_decompresses_to_the_fake_quant_weights(tmp_path, bits, sym, strategy):
    """compressed-tensors' own decompressor turns the written tensors back into (q - zp) * s,
    the fake-quantised weight, bit for bit with fp32 scales."""
    ct = pytest.importorskip("compressed_tensors")
    from compressed_tensors.compressors.pack_quantized.base import PackedQuantizationCompressor
    from compressed_tensors.quantization import QuantizationArgs, QuantizationConfig, QuantizationScheme

    g = torch.Generator().manual_seed(40 + bits)
    w = torch.randn(40, 384, generator=g) * 0.02
    w[torch.rand(40, 384, generator=g) < 0.002] *= 20
    entry, q, deq = _rtn_entry(w, bits, sym, strategy, 128)
    name = "model.layers.0.self_attn.q_proj.weight"
    state = CompressionState({name: deq, "model.norm.weight": torch.ones(384)})
    state.compressed[name] = entry
    cfg = CompressedTensorsWriter.save(state, str(tmp_path), scale_dtype=torch.float32,
                                       base_config={"model_type": "llama"}, ignore=["lm_head"])
    sd = load_safetensors(str(tmp_path / "model.safetensors"))
    assert torch.equal(sd["model.norm.weight"], torch.ones(384))
    mod = "model.layers.0.self_attn.q_proj"
    local = {k[len(mod) + 1:]: v for k, v in sd.items() if k.startswith(mod + ".")}
    assert set(local) == {"weight_packed", "weight_scale", "weight_shape"} | (set() if sym else {"weight_zero_point"})
    args = QuantizationArgs(num_bits=bits, type="int", symmetric=sym, strategy=strategy,
                            group_size=128 if strategy == "group" else None)
    out = PackedQuantizationCompressor.decompress(local, QuantizationScheme(targets=["Linear"], weights=args))
    zp = entry["zero_points"].to(torch.float32)
    s = entry["scales"]
    if strategy == "group":
        zp, s = zp.repeat_interleave(128, 1), s.repeat_interleave(128, 1)
    else:
        zp, s = zp.reshape(-1, 1), s.reshape(-1, 1)
    expect = (q.to(torch.float32) - zp) * s
    assert torch.equal(out["weight"].to(torch.float32), expect)
    with open(tmp_path / "config.json") as f:
        on_disk = json.load(f)
    assert on_disk == json.loads(json.dumps(cfg)) and on_disk["model_type"] == "llama"
    qc = QuantizationConfig.model_validate(on_disk["quantization_config"])
    grp = next(iter(qc.config_groups.values()))
    assert grp.targets == [mod] and grp.weights.num_bits == bits and grp.weights.symmetric == sym


def test_sparsity_config_records_2_4_masks(tmp_path):
    w = torch.randn(8, 16)
    mask = torch.zeros(8, 16, dtype=torch.uint8)
    mask.view(8, 4, 4)[:, :, :2] = 1
    state = CompressionState({"fc.weight": w * mask})
    state.compressed["fc.weight"] = {"mask": mask}
    cfg = CompressedTensorsWriter.save(state, str(tmp_path))
    sp = cfg["quantization_config"]["sparsity_config"]
    assert sp["sparsity_structure"] == "2:4" and sp["format"] == "dense" and abs(sp["global_sparsity"] - 0.5) < 1e-9
    assert sp["targets"] == ["fc"]
    assert torch.equal(load_safetensors(os.path.join(str(tmp_path), "model.safetensors"))["fc.weight"], w * mask)


def test_entries_from_pipeline_outputs():
    from llmcompressorsharp_b200.gptq import GPTQConfig

    cfg = GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128)
    layer = {"__stacked__mlp_in": {"codes": torch.zeros(1)},
             "gate_proj": {"codes": torch.zeros(4, 64, dtype=torch.uint8), "scales": torch.ones(4, 1),
                           "zero_points": torch.zeros(4, 1, dtype=torch.int32)}}
    e = CompressedTensorsWriter.entries_from_pipeline(layer, cfg, names=lambda n: f"model.layers.3.mlp.{n}.weight")
    assert list(e) == ["model.layers.3.mlp.gate_proj.weight"]
    assert e["model.layers.3.mlp.gate_proj.weight"]["num_bits"] == 4
    assert e["model.layers.3.mlp.gate_proj.weight"]["strategy"] == "group"


def test_vllm_reads_the_quantization_config():
    """vLLM's compressed-tensors config parser maps each written target to the W4A16 group
    scheme in pack-quantized format (config only: loading weights needs a GPU)."""
    pytest.importorskip("vllm")
    try:
        from vllm.model_executor.layers.quantization.compressed_tensors.compressed_tensors import (
            CompressedTensorsConfig)
    except Exception as e:  # noqa: BLE001 — vLLM's import can fail on hosts without its native parts
        pytest.skip(f"vLLM compressed-tensors config unavailable: {e}")
    entries = {f"model.layers.{i}.mlp.down_proj.weight": {"codes": torch.zeros(1), "num_bits": 4, "symmetric": False,
                                                          "strategy": "group", "group_size": 128} for i in range(2)}
    qc = CompressedTensorsWriter.quantization_config(entries, ignore=["lm_head"])
    cfg = CompressedTensorsConfig.from_config(qc)
    assert sorted(cfg.target_scheme_map) == ["model.layers.0.mlp.down_proj", "model.layers.1.mlp.down_proj"]
    args = cfg.target_scheme_map["model.layers.0.mlp.down_proj"]["weights"]
    strategy = getattr(args.strategy, "value", args.strategy)
    assert (args.num_bits, args.symmetric, args.group_size, strategy) == (4, False, 128, "group")
    assert cfg.target_scheme_map["model.layers.0.mlp.down_proj"]["format"] == "pack-quantized"
    assert cfg.ignore == ["lm_head"]


def test_ragged_last_group_keeps_ceil_groups():
    w = torch.randn(16, 320, generator=torch.Generator().manual_seed(3)) * 0.02
    entry, q, _ = _rtn_entry(w, 4, False, "group", 128)
    out = CompressedTensorsWriter.module_tensors("fc.weight", entry, w.shape, torch.float32)
    assert out["fc.weight_scale"].shape == (16, 3)
    assert out["fc.weight_packed"].shape == (16, 40)
    assert out["fc.weight_zero_point"].shape == (2, 3)
    assert out["fc.weight_shape"].tolist() == [16, 320]
    qs, _ = signed_codes(entry["codes"], entry["zero_points"], 4, False, 320, "group", 128)
    assert np.array_equal(qs.astype(np.int64), q.numpy().astype(np.int64) - 8)
