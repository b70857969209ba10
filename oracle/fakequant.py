"""Fake quantisation and int4 packing (oracle; test infrastructure only).

Restates:
  * ``FakeQuantize.Apply``               src/LLMCompressorSharp.TorchExtensions/Quantization/FakeQuantize.cs:22-38
  * ``FakeQuantizeFunction.forward``     src/LLMCompressorSharp.TorchExtensions/Quantization/FakeQuantizeFunction.cs:30-47
  * ``Int4PackedTensor``                 src/LLMCompressorSharp.TorchExtensions/Quantization/Int4PackedTensor.cs:17-162

The forward op chain is ``x.div(scale) -> round() -> add(zp) -> clamp(qmin, qmax) ->
sub(zp) -> mul(scale)``, every op in the INPUT dtype.  LibTorch computes each
reduced-precision (bf16/fp16) op in fp32 and rounds the result back to the dtype,
which ``_in_dtype`` restates; fp32 input is plain fp32 arithmetic.  ``div`` by a
scalar is true IEEE division on the CPU (not a reciprocal multiply).
"""

from __future__ import annotations

import numpy as np
import torch


def qrange(num_bits: int, symmetric: bool) -> tuple[int, int]:
    """FakeQuantize.cs:29-30 — symmetric [-(2^(b-1)-1), 2^(b-1)-1], asymmetric [0, 2^b-1]."""
    if num_bits < 2 or num_bits > 16:
        raise ValueError("numBits must be between 2 and 16 inclusive.")  # FakeQuantize.cs:24-28
    if symmetric:
        q = (1 << (num_bits - 1)) - 1
        return -q, q
    return 0, (1 << num_bits) - 1


def _in_dtype(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t if dtype == torch.float32 else t.to(dtype)


def fake_quantize_codes(x: torch.Tensor, scale, zp, num_bits: int, symmetric: bool):
    """Return (fake-quant tensor in x.dtype, integer codes as int32).

    ``scale``/``zp`` are scalars or tensors broadcastable to x (a per-row or per-group
    scale applied element-wise is identical to the reference's per-slice scalar calls,
    because every op is element-wise).  The integer code is the clamped value
    (FakeQuantizeFunction.cs:42), before the zero-point is subtracted again.
    """
    qmin, qmax = qrange(num_bits, symmetric)
    dt = x.dtype
    xf = x.to(torch.float32)
    s = torch.as_tensor(scale, dtype=torch.float32)
    z = torch.as_tensor(zp, dtype=torch.float32)
    t = _in_dtype(xf / s, dt).to(torch.float32)                # x.div(scale)        :39
    t = _in_dtype(torch.round(t), dt).to(torch.float32)        # .round()            :40
    t = _in_dtype(t + z, dt).to(torch.float32)                 # .add(zeroPoint)     :41
    t = _in_dtype(torch.clamp(t, qmin, qmax), dt).to(torch.float32)  # .clamp        :42
    codes = t.to(torch.int32)
    t = _in_dtype(t - z, dt).to(torch.float32)                 # .sub(zeroPoint)     :43
    out = _in_dtype(t * s, dt)                                 # .mul(scale)         :44
    return out.to(dt), codes


def fake_quantize(x: torch.Tensor, scale: float, zp: int, num_bits: int, symmetric: bool) -> torch.Tensor:
    """FakeQuantize.Apply (FakeQuantize.cs:22-38) with scalar scale / zero-point."""
    return fake_quantize_codes(x, scale, zp, num_bits, symmetric)[0]


def fake_quantize_torch_chain(x: torch.Tensor, scale: float, zp: int, num_bits: int, symmetric: bool) -> torch.Tensor:
    """The literal LibTorch op chain of FakeQuantizeFunction.forward (:39-44), used by the
    tests to confirm that ``fake_quantize`` restates it exactly for every dtype."""
    qmin, qmax = qrange(num_bits, symmetric)
    return x.div(scale).round().add(zp).clamp(qmin, qmax).sub(zp).mul(scale)


class Int4PackedTensor:
    """Int4PackedTensor.cs:17-162.

    Stores ``q - zp`` as signed bytes; packs two values per byte with the EVEN index in
    the HIGH nibble and the odd index in the low nibble (``v & 0xF``), ``(n+1)//2``
    bytes.  Unpacking sign-extends only when symmetric, so an asymmetric tensor whose
    ``q - zp`` is negative does not round-trip through the bytes: a property of the
    reference that is kept as-is.
    """

    def __init__(self, ints: np.ndarray, scale: float, zero_point: int, symmetric: bool):
        self.ints = ints.astype(np.int8)
        self.scale = np.float32(scale)
        self.zero_point = int(zero_point)
        self.symmetric = symmetric

    @property
    def element_count(self) -> int:
        return int(self.ints.size)

    @staticmethod
    def from_float(x: torch.Tensor, scale: float, zero_point: int, symmetric: bool) -> "Int4PackedTensor":
        """Int4PackedTensor.cs:79-100 — fp ops in x's dtype on the CPU, then int64."""
        qmin, qmax = (-7, 7) if symmetric else (0, 15)
        t = x.cpu().div(scale).round().add(zero_point).clamp(qmin, qmax).to(torch.int64)
        ints = (t.numpy().reshape(-1) - zero_point).astype(np.int8)  # (sbyte)(q - zp), :96
        return Int4PackedTensor(ints, scale, zero_point, symmetric)

    @property
    def packed_bytes(self) -> bytes:
        """Int4PackedTensor.cs:47-69."""
        n = self.ints.size
        out = np.zeros((n + 1) // 2, dtype=np.uint8)
        v = (self.ints.astype(np.int16) & 0x0F).astype(np.uint8)
        out[: (n + 1) // 2] = v[0::2] << 4
        out[: n // 2] |= v[1::2]
        return out.tobytes()

    @staticmethod
    def from_packed_bytes(packed: bytes, element_count: int, scale: float, zero_point: int,
                          symmetric: bool) -> "Int4PackedTensor":
        """Int4PackedTensor.cs:111-146."""
        b = np.frombuffer(packed, dtype=np.uint8)
        if b.size != (element_count + 1) // 2:
            raise ValueError(f"Expected {(element_count + 1) // 2} bytes for {element_count} int4 elements; got {b.size}.")
        idx = np.arange(element_count)
        nib = np.where(idx % 2 == 0, b[idx // 2] >> 4, b[idx // 2] & 0x0F).astype(np.int16)
        if symmetric:
            nib = np.where(nib & 0x08, nib - 16, nib)
        return Int4PackedTensor(nib.astype(np.int8), scale, zero_point, symmetric)

    def dequantize(self) -> torch.Tensor:
        """Int4PackedTensor.cs:152-161 — float(stored) * scale in fp32."""
        return torch.from_numpy((self.ints.astype(np.float32) * self.scale).astype(np.float32))


def pack_int4_rows(codes: torch.Tensor, zp: torch.Tensor | int = 0) -> torch.Tensor:
    """Row-wise int4 packing of a 2-D code matrix with the Int4PackedTensor byte layout
    (even column -> high nibble).  The stored nibble is ``(code - zp) & 0xF`` as in
    Int4PackedTensor.PackedBytes (:56); ``zp`` broadcasts per row/group.  Used for the
    packed output of the RTN/GPTQ entry points (extension; parity unpinned)."""
    c = codes.to(torch.int32) - torch.as_tensor(zp, dtype=torch.int32)
    v = (c & 0x0F).to(torch.uint8)
    m, n = v.shape
    if n % 2:
        v = torch.cat([v, torch.zeros(m, 1, dtype=torch.uint8)], dim=1)
    return (v[:, 0::2] << 4) | v[:, 1::2]
