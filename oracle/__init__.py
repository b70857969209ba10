"""CPU oracle for the one-shot compression hot path of LLMCompressorSharp.

TEST INFRASTRUCTURE ONLY.  This package is a plain PyTorch-CPU restatement of the
reference's C# code (TorchSharp 0.107 over LibTorch, which is the same op library
torch exposes here).  It exists to check the CUDA library, never to stand in for it:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it.  The product path
(``llmcompressorsharp_b200``) never imports, calls or links anything here.

Every function cites the reference file:line it restates.  Paths are relative to the
reference repository root (jamesburton/LLMCompressorSharp).

Pinning: the reference cannot be built or run in this environment (it needs the
.NET 10 SDK and the TorchSharp NuGet packages), so the oracle is pinned against the
known-answer values written in the reference's own xUnit tests (see
``tests/test_oracle_kats.py``, which ports each of them with a file:line citation).
Parts of the path that the reference does not implement (group-128 strategy,
SparseGPT, AWQ, packed int4 codes from a modifier) have no such values: for those the
oracle follows the reference's design documents and is marked "parity unpinned".
"""

from . import affine, fakequant, hessian, gptq, rtn, smoothquant, sparsegpt, awq  # noqa: F401
