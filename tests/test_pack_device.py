"""compressed-tensors pack-quantized words packed on the device (llmc_pack_compressed_tensors)
against the host packing of output.py (signed_codes + pack_int32), which compressed-tensors'
own decompressor is checked against in test_output.py.  Byte-exact, for codes written by the
CUDA RTN and GPTQ paths, ragged shapes included."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def host_words(codes, zps, m, n, bits, sym, strategy, gs):
    from llmcompressorsharp_b200.output import pack_int32, signed_codes

    q, zp = signed_codes(codes.cpu(), zps.cpu(), bits, sym, n, strategy, gs)
    packed = torch.from_numpy(pack_int32(q, bits))
    zw = None
    if not sym and strategy in ("group", "channel"):
        zw = torch.from_numpy(pack_int32(zp.reshape(m, -1), bits, packed_dim=0))
    return packed, zw


@pytest.mark.parametrize("bits,sym", [(4, False), (4, True), (8, False), (8, True)])
@pytest.mark.parametrize("strategy", ["group", "channel", "tensor"])
@pytest.mark.parametrize("m,n", [(96, 512), (37, 300)])
def test_device_packing_equals_host_packing_rtn(bits, sym, strategy, m, n):
    from llmcompressorsharp_b200 import RtnConfig, rtn_quantize
    from llmcompressorsharp_b200.output import pack_on_device

    gs = 128 if n % 128 == 0 else 100
    w = (torch.randn(m, n, generator=torch.Generator().manual_seed(m + n + bits)) * 0.02).to(torch.bfloat16)
    _, codes, scales, zps = rtn_quantize(w.to(DEV), RtnConfig(num_bits=bits, symmetric=sym, strategy=strategy,
                                                               group_size=gs))
    packed, zw = pack_on_device(codes, zps, m, n, bits, sym, strategy, gs)
    hp, hz = host_words(codes, zps, m, n, bits, sym, strategy, gs)
    assert torch.equal(packed.cpu(), hp)
    if hz is None:
        assert zw is None
    else:
        assert torch.equal(zw.cpu(), hz)


def test_writer_device_and_host_paths_write_the_same_tensors():
    from llmcompressorsharp_b200 import GPTQConfig, gptq_quantize_u
    from llmcompressorsharp_b200.output import CompressedTensorsWriter

    m, n = 128, 640
    g = torch.Generator().manual_seed(9)
    w = (torch.randn(m, n, generator=g) * 0.02).to(torch.bfloat16)
    cfg = GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128)
    res = gptq_quantize_u(w.to(DEV), torch.eye(n, device=DEV), cfg)
    entry = {"codes": res.codes, "scales": res.scales, "zero_points": res.zero_points, "num_bits": 4,
             "symmetric": False, "strategy": "group", "group_size": 128}
    dev_t = CompressedTensorsWriter.module_tensors("layer.weight", entry, (m, n), torch.float32)
    host_entry = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in entry.items()}
    host_t = CompressedTensorsWriter.module_tensors("layer.weight", host_entry, (m, n), torch.float32)
    assert set(dev_t) == set(host_t)
    for k in dev_t:
        assert torch.equal(dev_t[k], host_t[k]), k


def test_packing_rejects_bad_arguments():
    import ctypes as C

    from llmcompressorsharp_b200 import _lib
    from llmcompressorsharp_b200.errors import LlmcError

    codes = torch.zeros(4, 8, dtype=torch.uint8, device=DEV)
    out = torch.empty(4, 2, dtype=torch.int32, device=DEV)
    with pytest.raises(LlmcError):  # 5 bits do not divide a 32-bit word
        _lib.call("llmc_pack_compressed_tensors", C.c_void_p(_lib.ctx_for(0)), _lib.ptr(codes), C.c_int64(4),
                  C.c_int64(8), C.c_int64(8), _lib.ptr(None), C.c_int32(1), C.c_int64(8), C.c_int32(5), C.c_int32(1),
                  _lib.ptr(out), C.c_int64(2), _lib.ptr(None))
