"""Host-side fault injection through the C ABI (LLMC_FAULT), on CPU: an entry point told to
fail returns the injected status without touching its arguments or the GPU, the Python layer
maps it to the reference's exception type, and a CompressionSession whose modifier hits it
ends FAILED and still finalises (CompressionSession.cs:56-99).  No GPU is faulted: the
failures are made on the host."""

import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(code: str, fault: str | None) -> str:
    env = dict(os.environ)
    env.pop("LLMC_FAULT", None)
    if fault is not None:
        env["LLMC_FAULT"] = fault
    r = subprocess.run([sys.executable, "-c", textwrap.dedent(code)], capture_output=True, text=True, env=env,
                       cwd=ROOT, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return r.stdout


CALLS = """
import ctypes as C
from llmcompressorsharp_b200 import _lib
lib = _lib.load()
for name, args in CASES:
    st = getattr(lib, name)(*args)
    print(name, st, _lib.last_error())
"""


def test_injected_status_replaces_the_call():
    code = "CASES = [('llmc_hessian_update', (None, None, 0, 1, 1)), ('llmc_hessian_reset', (None,)), " \
           "('llmc_sync', (None,))]\n" + CALLS
    plain = _run(code, None).splitlines()
    assert plain[0].startswith("llmc_hessian_update 1 ") and "must not be null" in plain[0]
    out = _run(code, "llmc_hessian_update:5,llmc_sync:7").splitlines()
    assert out[0] == "llmc_hessian_update 5 injected fault in llmc_hessian_update (call 1)"
    assert out[1].startswith("llmc_hessian_reset 1 ")  # not named: the real argument check runs
    assert out[2] == "llmc_sync 7 injected fault in llmc_sync (call 1)"


def test_injection_on_the_kth_call_only():
    code = "CASES = [('llmc_hessian_reset', (None,))] * 4\n" + CALLS
    out = _run(code, "llmc_hessian_reset:4:2").splitlines()
    assert [int(line.split()[1]) for line in out] == [1, 4, 1, 1]
    assert "(call 2)" in out[1]


def test_malformed_specs_are_ignored():
    code = "CASES = [('llmc_hessian_reset', (None,))]\n" + CALLS
    out = _run(code, "bogus,llmc_hessian_reset:99,llmc_hessian_reset:-3,:5,llmc_hessian_reset:x").splitlines()
    assert out[0].startswith("llmc_hessian_reset 1 ")


def test_python_layer_raises_the_mapped_exception():
    code = """
    import ctypes as C
    from llmcompressorsharp_b200 import _lib
    from llmcompressorsharp_b200.errors import CudaError, NotPositiveDefiniteError, TimeoutError_
    for name, cls in (("llmc_sync", CudaError), ("llmc_hessian_reset", NotPositiveDefiniteError),
                      ("llmc_launch_count", TimeoutError_)):
        try:
            _lib.call(name, None) if name != "llmc_launch_count" else _lib.call(name, None, None)
        except cls as e:
            print(name, type(e).__name__, e.status, "injected" in str(e))
    """
    out = _run(code, "llmc_sync:5,llmc_hessian_reset:4,llmc_launch_count:7").splitlines()
    assert out == ["llmc_sync CudaError 5 True", "llmc_hessian_reset NotPositiveDefiniteError 4 True",
                   "llmc_launch_count TimeoutError_ 7 True"]


def test_session_fails_and_finalises_on_an_injected_fault():
    """A modifier whose OnEnd reaches a C-ABI call that is told to fail: the session records
    the mapped exception, ends FAILED and still finalises every initialised modifier."""
    code = """
    import torch
    from llmcompressorsharp_b200 import _lib
    from llmcompressorsharp_b200.session import CompressionSession, CompressionState, ModifierBase

    class Calling(ModifierBase):
        def __init__(self, name):
            super().__init__(name)
            self.finalized = False

        def on_end_core(self, state):
            _lib.call("llmc_hessian_reset", None)

        def on_finalize_core(self, state):
            self.finalized = True

    mods = [Calling("a"), Calling("b")]
    session = CompressionSession(mods)
    status = session.run(CompressionState({"fc.weight": torch.zeros(2, 2)}), [torch.zeros(1)])
    print(status.name, type(session.failure).__name__, "injected fault" in str(session.failure),
          all(m.finalized for m in mods))
    """
    assert _run(code, "llmc_hessian_reset:5").splitlines()[-1] == "FAILED CudaError True True"
    assert _run(code, None).splitlines()[-1] == "FAILED ArgumentError False True"
