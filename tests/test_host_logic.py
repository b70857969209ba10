"""Host-side control flow that needs no GPU: modifier lifecycle, session failure handling,
target matching (ModifierBaseTests.cs, CompressionSessionTests.cs, TargetMatcherTests.cs)."""

import pytest
import torch

from llmcompressorsharp_b200.session import (CompressionSession, CompressionState, ModifierBase,
                                             ModifierLifecycleError, SessionStatus, TargetMatcher)


class Recording(ModifierBase):
    def __init__(self, log, fail_on=None):
        super().__init__("rec")
        self.log = log
        self.fail_on = fail_on

    def _rec(self, what):
        self.log.append(what)
        if what == self.fail_on:
            raise RuntimeError("boom")

    def on_initialize(self, state):
        self._rec("init")

    def on_start_core(self, state):
        self._rec("start")

    def on_batch_core(self, state):
        self._rec(f"batch{state.current_batch_index}")

    def on_end_core(self, state):
        self._rec("end")

    def on_finalize_core(self, state):
        self._rec("final")


def test_session_lifecycle_order():  # CompressionSessionTests.cs
    log = []
    st = CompressionState({"w": torch.zeros(1)})
    s = CompressionSession([Recording(log)])
    assert s.run(st, [1, 2]) == SessionStatus.COMPLETED
    assert log == ["init", "start", "batch0", "batch1", "end", "final"]
    with pytest.raises(ModifierLifecycleError):
        s.run(st, [])


def test_session_failure_still_finalizes():  # CompressionSession.cs:91-99
    log = []
    s = CompressionSession([Recording(log, fail_on="batch1")])
    assert s.run(CompressionState({}), [1, 2, 3]) == SessionStatus.FAILED
    assert isinstance(s.failure, RuntimeError)
    assert log[-1] == "final" and "end" not in log


def test_modifier_guards():  # ModifierBase.cs:47-116
    m = Recording([])
    st = CompressionState({})
    with pytest.raises(ModifierLifecycleError):
        m.on_start(st)
    m.initialize(st)
    with pytest.raises(ModifierLifecycleError):
        m.initialize(st)
    with pytest.raises(ModifierLifecycleError):
        m.on_batch(st)
    m.on_start(st)
    m.on_end(st)
    with pytest.raises(ModifierLifecycleError):
        m.on_batch(st)
    m.finalize(st)
    with pytest.raises(ModifierLifecycleError):
        m.finalize(st)


def test_target_matcher():  # TargetMatcher.cs:22-86
    names = ["model.layer.0.q_proj.weight", "model.lm_head.weight", "fc.weight"]
    assert TargetMatcher.filter(names, [], []) == names
    assert TargetMatcher.filter(names, ["model.layer.*"], ["*.lm_head.*"]) == ["model.layer.0.q_proj.weight"]
    assert TargetMatcher.filter(names, ["fc.weight"], []) == ["fc.weight"]
    assert TargetMatcher.filter(names, ["*"], ["*.weight"]) == []


def test_rtn_config_rejects_token():
    from llmcompressorsharp_b200.errors import NotSupportedError
    from llmcompressorsharp_b200.rtn import RtnConfig

    with pytest.raises(NotSupportedError):
        RtnConfig(strategy="token").to_c()


def test_gptq_config_defaults():  # GPTQConfig.cs:22-59, GPTQConfigTests.cs:16-56
    from llmcompressorsharp_b200.gptq import GPTQConfig

    c = GPTQConfig()
    assert (c.num_bits, c.symmetric, c.strategy, c.channel_axis, c.block_size, c.act_order) == (4, True, "channel", 0,
                                                                                                 128, False)
    assert abs(c.dampening_frac - 0.01) < 1e-9
    q = c.to_c()
    assert q.num_bits == 4 and q.strategy == 1 and q.block_size == 128


def test_chunk_waits():
    """Which copy mark each Hessian update chunk waits for (pipeline.chunk_waits)."""
    from llmcompressorsharp_b200.pipeline import chunk_waits

    assert chunk_waits([], 10, 4) == [-1, -1, -1]
    assert chunk_waits([4, 8, 10], 10, 4) == [0, 1, 2]
    assert chunk_waits([10], 10, 4) == [0, -1, -1]
    # marks every 3000 rows, chunks of 4096 rows: chunk 0 needs rows 4096 -> mark 1 (6000)
    assert chunk_waits([3000, 6000, 9000, 10000], 10000, 4096) == [1, 2, 3]
    # marks finer than chunks and one mark short of the end: the last mark covers the rest
    assert chunk_waits([1, 2, 3, 4, 5], 12, 4) == [3, 4, -1]


def test_site_order_widest_first_and_stable():
    """The overlapped schedule's site order (GptqPipeline.site_order): widest first, ties in the
    model's order, so every rank of a distributed job issues its reductions in the same order."""
    from types import SimpleNamespace

    from llmcompressorsharp_b200.pipeline import GptqPipeline, llama_sites

    sites = llama_sites(4096, 14336, 32, 8)
    order = [s.name for s in GptqPipeline.site_order(SimpleNamespace(sites=sites))]
    assert order == ["down_in", "attn_in", "o_in", "mlp_in"]
    wide = llama_sites(8192, 4096, 64, 8)  # intermediate narrower than hidden
    assert [s.name for s in GptqPipeline.site_order(SimpleNamespace(sites=wide))] == ["attn_in", "o_in", "mlp_in",
                                                                                        "down_in"]


class _CountingAccumulator:
    """Stands in for HessianAccumulator (which needs the GPU) where only the hook path is tested."""

    def __init__(self, in_features):
        self.in_features = in_features
        self.sample_count = 0

    def update(self, x):
        assert x.shape[-1] == self.in_features
        self.sample_count += x.numel() // self.in_features


def test_activation_hooks():  # ActivationHookManagerTests.cs:22-117
    from llmcompressorsharp_b200.errors import ArgumentError
    from llmcompressorsharp_b200.hessian import ActivationHookManager

    lin = torch.nn.Linear(4, 2)
    acc = _CountingAccumulator(4)
    mgr = ActivationHookManager()
    mgr.register_for(lin, acc)
    lin(torch.tensor([[1.0, 2.0, 3.0, 4.0]]))
    assert acc.sample_count == 1  # :22-36
    l1, l2 = torch.nn.Linear(3, 4), torch.nn.Linear(4, 2)
    a1, a2 = _CountingAccumulator(3), _CountingAccumulator(4)
    mgr.register_for(l1, a1)
    mgr.register_for(l2, a2)
    l2(l1(torch.tensor([[1.0, 2.0, 3.0]])))
    assert (a1.sample_count, a2.sample_count) == (1, 1)  # :38-56
    mgr.clear()  # :78-99: cleared hooks stop, re-registration works
    lin(torch.ones(1, 4))
    assert acc.sample_count == 1
    mgr.register_for(lin, acc)
    lin(torch.ones(1, 4))
    assert acc.sample_count == 2
    mgr.dispose()  # :58-76
    lin(torch.ones(1, 4))
    assert acc.sample_count == 2
    with pytest.raises(ArgumentError):  # :101-117
        ActivationHookManager().register_for(None, acc)
    with pytest.raises(ArgumentError):
        ActivationHookManager().register_for(lin, None)


def test_forward_hook_handle():  # ForwardHookHandleTests.cs:14-40
    from llmcompressorsharp_b200.errors import ArgumentError
    from llmcompressorsharp_b200.hessian import ForwardHookHandle

    calls = []
    h = ForwardHookHandle(lambda: calls.append(1))
    h.dispose()
    h.dispose()
    assert calls == [1]
    with pytest.raises(ArgumentError):
        ForwardHookHandle(None)
