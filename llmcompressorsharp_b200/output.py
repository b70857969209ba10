"""Output writers: the reference's dense safetensors file and a compressed-tensors checkpoint.

``SafetensorsWriter`` mirrors src/LLMCompressorSharp.Core/Output/SafetensorsWriter.cs:19-57:
``save(state, path)`` writes ``state.named_weights`` (the fake-quantised weights the modifiers
leave there) under their names, ``load(path)`` reads a file back.

``CompressedTensorsWriter`` writes what the reference's documentation names as the output
format (docs/llm-compressor/deployment.md:124-132) and the reference itself does not produce:
the packed integer weights with their scales and zero-points in safetensors, plus the
``quantization_config`` block of ``config.json``, in the layout of compressed-tensors'
``pack-quantized`` format:

- ``<module>.weight_packed``  int32 [out, ceil(in / (32 / bits))]: signed codes q' offset by
  2^(bits-1), packed low bits first (element i of a word at bits [i*bits, (i+1)*bits));
- ``<module>.weight_scale``   [out, groups] (group), [out, 1] (channel) or [1] (tensor);
- ``<module>.weight_zero_point`` (asymmetric only) int32 [ceil(out / (32 / bits)), groups],
  signed zero-points packed the same way along the output dimension (tensor strategy: int8 [1]);
- ``<module>.weight_shape``   int64 [2].

The library's codes follow the reference's conventions (FakeQuantize.cs:29-30): symmetric
q in [-(2^(b-1)-1), 2^(b-1)-1] with zero-point 0, asymmetric q in [0, 2^b-1] with
zero-point in the same range; int4 codes are stored as (q - zp) & 0xF, two per byte, even
column in the high nibble (Int4PackedTensor.cs:47-69).  compressed-tensors keeps signed
codes for both, so asymmetric codes and zero-points move down by 2^(b-1); (q' - zp') * s is
unchanged, so the dequantised weight is the same.

A weight whose in_features is not a multiple of the group size keeps its ragged last group:
``weight_scale`` has ceil(in / group) columns.  Readers that infer the group size from the
shapes (compressed-tensors' argument-free ``dequantize``) need in_features divisible by the
group size; the ``quantization_config`` states the group size for the others.

SparseGPT masks are recorded as a ``sparsity_config`` (dense format, the pruned weights are
written as they are).  Codes that are CUDA tensors are packed on the device
(``llmc_pack_compressed_tensors``, ``pack_on_device``), so only the packed words cross PCIe;
host codes take the numpy path (``signed_codes`` + ``pack_int32``), which produces the same
words.
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np
import torch

from .errors import ArgumentError

_ST_DTYPES = {
    torch.float64: "F64", torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16",
    torch.int64: "I64", torch.int32: "I32", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8",
    torch.bool: "BOOL",
}
_ST_FROM = {v: k for k, v in _ST_DTYPES.items()}


# --------------------------------------------------------------------------- safetensors
def save_safetensors(tensors: dict, path: str, metadata: dict | None = None) -> None:
    """Write ``tensors`` (name -> tensor, any device) as a safetensors file: an 8-byte
    little-endian header length, a JSON header of dtype / shape / byte offsets (8-byte aligned
    total), then the raw little-endian bytes in name order."""
    if not path or not str(path).strip():
        raise ArgumentError("path must not be empty")
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if t.dtype not in _ST_DTYPES:
            raise ArgumentError(f"{name}: dtype {t.dtype} has no safetensors code")
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _ST_DTYPES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * ((8 - len(hb) % 8) % 8)
    tmp = str(path) + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def load_safetensors(path: str) -> dict:
    """Read a safetensors file into CPU tensors (name -> tensor)."""
    if not path or not str(path).strip():
        raise ArgumentError("path must not be empty")
    if not os.path.exists(path):
        raise FileNotFoundError(f"Safetensors file not found: {path}")
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n).decode("utf-8"))
        data = f.read()
    out = {}
    for name, spec in header.items():
        if name == "__metadata__":
            continue
        a, b = spec["data_offsets"]
        dt = _ST_FROM[spec["dtype"]]
        buf = bytearray(data[a:b])
        t = torch.frombuffer(buf, dtype=torch.uint8) if b > a else torch.empty(0, dtype=torch.uint8)
        out[name] = t.view(dt).reshape(spec["shape"]).clone()
    return out


class SafetensorsWriter:
    """SafetensorsWriter.cs:19-57."""

    @staticmethod
    def save(state, path: str) -> None:
        if state is None:
            raise ArgumentError("state must not be null")
        save_safetensors(state.named_weights, path)

    @staticmethod
    def load(path: str) -> dict:
        return load_safetensors(path)


# --------------------------------------------------------------------------- packing
def signed_codes(codes: torch.Tensor, zero_points: torch.Tensor, num_bits: int, symmetric: bool, n: int,
                 strategy: str, group_size: int) -> tuple[np.ndarray, np.ndarray]:
    """The library's codes of one [m, n] weight as compressed-tensors' signed codes q' (int8
    [m, n]) and zero-points zp' (int8, the zero-point tensor's shape)."""
    c = codes.detach().cpu().numpy()
    zp = zero_points.detach().cpu().numpy().astype(np.int64)
    m = c.shape[0]
    half = 1 << (num_bits - 1)
    if strategy == "group":
        zfull = np.repeat(zp.reshape(m, -1), group_size, axis=1)[:, :n]
    elif strategy == "channel":
        zfull = np.broadcast_to(zp.reshape(m, 1), (m, n))
    else:
        zfull = np.full((m, n), int(zp.reshape(-1)[0]))
    if num_bits <= 4:
        # (q - zp) & 0xF, even column in the high nibble
        nib = np.empty((m, 2 * c.shape[1]), dtype=np.int64)
        nib[:, 0::2] = c >> 4
        nib[:, 1::2] = c & 0xF
        nib = nib[:, :n]
        mod = 1 << num_bits
        if symmetric:  # q = sign-extended nibble (|q| < 2^(b-1))
            q = np.where(nib & 0x8, nib - 16, nib)
        else:  # q in [0, 2^b - 1] is a full residue system: q = (nibble + zp) mod 2^b
            q = (nib + zfull) % mod
    else:
        raw = c[:, :n].astype(np.int64)
        q = np.where(raw > 127, raw - 256, raw) if symmetric else raw
    if symmetric:
        return q.astype(np.int8), np.zeros(zp.shape, dtype=np.int8)
    return (q - half).astype(np.int8), (zp - half).astype(np.int8)


def pack_int32(values: np.ndarray, num_bits: int, packed_dim: int = 1) -> np.ndarray:
    """Signed int8 values [r, c] -> int32 words: value + 2^(bits-1) in `bits`-wide fields,
    32 / bits per word, first element in the low bits, packed along `packed_dim` (zero padded)."""
    v = values.astype(np.int64) + (1 << (num_bits - 1))
    if packed_dim == 0:
        v = v.T
    per = 32 // num_bits
    r, c = v.shape
    cp = -(-c // per) * per
    if cp != c:
        v = np.pad(v, ((0, 0), (0, cp - c)))
    v = v.reshape(r, cp // per, per).astype(np.uint64)
    word = np.zeros((r, cp // per), dtype=np.uint64)
    for i in range(per):
        word |= v[:, :, i] << np.uint64(i * num_bits)
    out = word.astype(np.uint32).view(np.int32)
    return out.T.copy() if packed_dim == 0 else out


def pack_on_device(codes: torch.Tensor, zero_points: torch.Tensor, m: int, n: int, num_bits: int, symmetric: bool,
                   strategy: str, group_size: int):
    """``weight_packed`` (int32 [m, ceil(n / (32 / bits))]) and, for asymmetric channel / group
    weights, the row-packed ``weight_zero_point`` of one weight whose codes and zero-points are
    on a CUDA device; the same words as ``pack_int32(signed_codes(...))``.  Returns (packed,
    packed zero-points or None), both on the codes' device."""
    import ctypes as C

    from . import _lib
    from ._device import ctx

    dev = codes.device
    c = codes.detach().contiguous()
    z = zero_points.detach().to(device=dev, dtype=torch.int32).contiguous()
    per = 32 // num_bits
    packed = torch.empty(m, -(-n // per), dtype=torch.int32, device=dev)
    zp_packed = None
    if not symmetric and strategy in ("group", "channel"):
        g = -(-n // group_size) if strategy == "group" else 1
        zp_packed = torch.empty(-(-m // per), g, dtype=torch.int32, device=dev)
    _lib.call("llmc_pack_compressed_tensors", C.c_void_p(ctx(dev)), _lib.ptr(c), C.c_int64(m), C.c_int64(n),
              C.c_int64(c.shape[1]), _lib.ptr(z), C.c_int32(_lib.STRATEGY[strategy]), C.c_int64(group_size),
              C.c_int32(num_bits), C.c_int32(int(symmetric)), _lib.ptr(packed), C.c_int64(packed.shape[1]),
              _lib.ptr(zp_packed))
    return packed, zp_packed


class CompressedTensorsWriter:
    """compressed-tensors ``pack-quantized`` checkpoint from a CompressionState."""

    @staticmethod
    def module_tensors(name: str, entry: dict, shape, scale_dtype: torch.dtype) -> dict:
        """Tensors of one quantised weight named ``name`` (``<module>.weight``)."""
        module = name[: -len(".weight")] if name.endswith(".weight") else name
        bits, sym, strat, gs = entry["num_bits"], entry["symmetric"], entry["strategy"], entry["group_size"]
        if bits not in (4, 8):
            raise ArgumentError(f"{name}: pack-quantized needs 4 or 8 bits (got {bits})")
        m, n = int(shape[0]), int(shape[-1])
        codes = entry["codes"]
        if torch.is_tensor(codes) and codes.is_cuda:
            packed, zp_words = pack_on_device(codes, entry["zero_points"], m, n, bits, sym, strat, gs)
            packed, zp_words = packed.cpu(), (zp_words.cpu() if zp_words is not None else None)
            zp = (entry["zero_points"].detach().cpu().numpy().astype(np.int64) - (1 << (bits - 1))).astype(np.int8)
        else:
            q, zp = signed_codes(codes, entry["zero_points"], bits, sym, n, strat, gs)
            packed = torch.from_numpy(pack_int32(q, bits))
            zp_words = None
        scales = entry["scales"].detach().cpu().to(torch.float32)
        if strat == "group":
            scales = scales.reshape(m, -1)
        elif strat == "channel":
            scales = scales.reshape(m, 1)
        else:
            scales = scales.reshape(1)
        out = {f"{module}.weight_packed": packed,
               f"{module}.weight_scale": scales.to(scale_dtype),
               f"{module}.weight_shape": torch.tensor([m, n], dtype=torch.int64)}
        if not sym:
            if strat in ("group", "channel"):
                out[f"{module}.weight_zero_point"] = (zp_words if zp_words is not None else
                                                      torch.from_numpy(pack_int32(zp.reshape(m, -1), bits, packed_dim=0)))
            else:
                out[f"{module}.weight_zero_point"] = torch.from_numpy(zp.reshape(1).astype(np.int8))
        return out

    @staticmethod
    def quantization_config(entries: dict, ignore=None) -> dict:
        """The ``quantization_config`` block: one config group per distinct weight scheme."""
        groups, seen = {}, {}
        for name, e in entries.items():
            if "codes" not in e:
                continue
            key = (e["num_bits"], e["symmetric"], e["strategy"], e["group_size"] if e["strategy"] == "group" else None)
            if key not in seen:
                seen[key] = f"group_{len(seen)}"
                groups[seen[key]] = {
                    "targets": [], "format": "pack-quantized",
                    "weights": {"num_bits": key[0], "type": "int", "symmetric": bool(key[1]), "strategy": key[2],
                                "group_size": key[3], "dynamic": False, "observer": "minmax", "actorder": None,
                                "block_structure": None, "observer_kwargs": {}},
                    "input_activations": None, "output_activations": None}
            module = name[: -len(".weight")] if name.endswith(".weight") else name
            groups[seen[key]]["targets"].append(module)
        return {"quant_method": "compressed-tensors", "format": "pack-quantized" if groups else "dense",
                "quantization_status": "compressed", "config_groups": groups, "ignore": list(ignore or []),
                "kv_cache_scheme": None}

    @staticmethod
    def entries_from_pipeline(layer_outputs: dict, cfg, names=None) -> dict:
        """``state.compressed``-style entries from one layer's ``GptqPipeline`` outputs
        (weight name -> {codes, scales, zero_points}), with the scheme of the GPTQConfig
        ``cfg``; ``names`` maps the pipeline's weight names to checkpoint names (default:
        unchanged)."""
        out = {}
        for wname, o in layer_outputs.items():
            if wname.startswith("__stacked__") or "codes" not in o:
                continue
            key = names(wname) if callable(names) else (names or {}).get(wname, wname)
            out[key] = {"codes": o["codes"], "scales": o["scales"], "zero_points": o["zero_points"],
                        "num_bits": cfg.num_bits, "symmetric": cfg.symmetric, "strategy": cfg.strategy,
                        "group_size": cfg.group_size}
        return out

    @staticmethod
    def sparsity_config(entries: dict) -> dict | None:
        masked = [n for n, e in entries.items() if "mask" in e]
        if not masked:
            return None
        structure = "unstructured"
        for n in masked:
            m = entries[n]["mask"].detach().cpu()
            if m.dim() == 2 and m.shape[1] % 4 == 0 and bool((m.reshape(m.shape[0], -1, 4).sum(-1) == 2).all()):
                structure = "2:4"
            else:
                structure = "unstructured"
                break
        total = sum(entries[n]["mask"].numel() for n in masked)
        kept = sum(int(entries[n]["mask"].detach().cpu().to(torch.int64).sum()) for n in masked)
        return {"format": "dense", "sparsity_structure": structure, "global_sparsity": 1.0 - kept / max(1, total),
                "targets": [n[: -len(".weight")] if n.endswith(".weight") else n for n in masked], "ignore": []}

    @classmethod
    def save(cls, state, out_dir: str, scale_dtype: torch.dtype = torch.bfloat16, base_config: dict | None = None,
             ignore=None) -> dict:
        """Write ``model.safetensors`` and ``config.json`` under ``out_dir``: quantised weights
        packed, every other weight dense in its dtype.  Returns the written config."""
        if state is None:
            raise ArgumentError("state must not be null")
        if not out_dir or not str(out_dir).strip():
            raise ArgumentError("out_dir must not be empty")
        os.makedirs(out_dir, exist_ok=True)
        tensors = {}
        for name, w in state.named_weights.items():
            e = state.compressed.get(name)
            if e is not None and "codes" in e and e.get("codes") is not None:
                tensors.update(cls.module_tensors(name, e, w.shape, scale_dtype))
            else:
                tensors[name] = w
        save_safetensors(tensors, os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
        cfg = dict(base_config or {})
        cfg["quantization_config"] = cls.quantization_config(state.compressed, ignore)
        sp = cls.sparsity_config(state.compressed)
        if sp is not None:
            cfg["quantization_config"]["sparsity_config"] = sp
        with open(os.path.join(out_dir, "config.json"), "w") as f:
            json.dump(cfg, f, indent=2)
        return cfg
