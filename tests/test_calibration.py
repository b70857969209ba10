"""The calibration forward on CPU: a small random-initialised LLaMA, its module names, and
``drive`` feeding hooks inside a CompressionSession (a recording accumulator stands in for
the device Hessian)."""

import torch

from llmcompressorsharp_b200.calibration import SHAPES, LlamaForCalibration, LlamaShape, calibration_batches, drive
from llmcompressorsharp_b200.hessian import ActivationHookManager
from llmcompressorsharp_b200.session import CompressionSession, CompressionState, ModifierBase

TINY = LlamaShape(hidden=64, intermediate=96, heads=4, kv_heads=2, layers=2, vocab=101)


def test_presets_match_the_job_shapes():
    s = SHAPES["llama-3-8b"]
    assert (s.hidden, s.intermediate, s.heads, s.kv_heads, s.layers) == (4096, 14336, 32, 8, 32)
    s = SHAPES["smollm2-135m"]
    assert (s.hidden, s.intermediate, s.heads, s.kv_heads, s.layers, s.vocab) == (576, 1536, 9, 3, 30, 49152)
    assert SHAPES["llama-3-70b"].intermediate == 28672


def test_model_names_shapes_and_seed():
    m = LlamaForCalibration(TINY, dtype=torch.float32, seed=3)
    names = sorted(m.linear_modules())
    assert "model.layers.0.self_attn.q_proj" in names and "model.layers.1.mlp.down_proj" in names
    assert len(names) == 7 * TINY.layers
    w = m.linear_weights()
    assert w["model.layers.0.self_attn.k_proj.weight"].shape == (TINY.kv_heads * TINY.head_dim, TINY.hidden)
    assert w["model.layers.1.mlp.down_proj.weight"].shape == (TINY.hidden, TINY.intermediate)
    again = LlamaForCalibration(TINY, dtype=torch.float32, seed=3)
    assert all(torch.equal(a, b) for a, b in zip(w.values(), again.linear_weights().values()))
    assert abs(float(w["model.layers.0.mlp.up_proj.weight"].std()) - 0.02) < 0.005


def test_forward_is_causal():
    m = LlamaForCalibration(TINY, dtype=torch.float32, seed=4)
    ids = next(calibration_batches(TINY.vocab, 2, 12, 2, seed=5))
    y = m(ids)
    assert y.shape == (2, 12, TINY.hidden) and torch.isfinite(y).all()
    ids2 = ids.clone()
    ids2[:, 8:] = (ids2[:, 8:] + 1) % TINY.vocab
    y2 = m(ids2)
    assert torch.allclose(y[:, :8], y2[:, :8], atol=1e-5)
    assert not torch.allclose(y[:, 8:], y2[:, 8:])


def test_calibration_batches_are_seeded_and_sized():
    a = list(calibration_batches(50, 7, 5, 3, seed=9))
    b = list(calibration_batches(50, 7, 5, 3, seed=9))
    assert [t.shape for t in a] == [(3, 5), (3, 5), (1, 5)]
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    assert all(int(t.min()) >= 0 and int(t.max()) < 50 for t in a)


class _Recorder:
    def __init__(self):
        self.rows = 0
        self.d = None

    def update(self, x):
        self.d = x.shape[-1]
        self.rows += x.reshape(-1, x.shape[-1]).shape[0]


class _RecordingModifier(ModifierBase):
    """Attaches hooks in OnStart like GPTQModifier and checks in OnBatch that the caller's
    forward has already fired them for the current batch."""

    def __init__(self):
        super().__init__("record")
        self.acc = {}
        self.seen = []

    def on_start_core(self, state):
        self.hooks = ActivationHookManager()
        for name, mod in state.named_modules.items():
            self.acc[name] = _Recorder()
            self.hooks.register_for(mod, self.acc[name])

    def on_batch_core(self, state):
        self.seen.append(self.acc["model.layers.0.self_attn.q_proj"].rows)

    def on_end_core(self, state):
        self.hooks.dispose()


def test_drive_fires_the_hooks_before_each_batch_reaches_the_session():
    m = LlamaForCalibration(TINY, dtype=torch.float32, seed=6)
    batches = list(calibration_batches(TINY.vocab, 5, 8, 2, seed=7))
    state = CompressionState(m.linear_weights())
    state.named_modules = m.linear_modules()
    mod = _RecordingModifier()
    session = CompressionSession([mod])
    status = session.run(state, drive(m, batches))
    assert status.name == "COMPLETED", session.failure
    assert mod.seen == [16, 32, 40]  # rows seen by the time each batch reaches OnBatch (2, 2, 1 sequences of 8)
    tokens = 5 * 8
    for name, acc in mod.acc.items():
        assert acc.rows == tokens, name
        want = TINY.intermediate if name.endswith("down_proj") else TINY.hidden
        assert acc.d == want, name


def test_forward_matches_the_transformers_llama():
    """With the same weights, the calibration model's output equals transformers' LlamaModel
    (last hidden state after the final norm), so the activations reaching the hooks are a
    standard LLaMA's."""
    tr = __import__("pytest").importorskip("transformers")
    s = LlamaShape(hidden=64, intermediate=96, heads=4, kv_heads=2, layers=2, vocab=101, rope_theta=10000.0)
    ours = LlamaForCalibration(s, dtype=torch.float32, seed=3)
    cfg = tr.LlamaConfig(hidden_size=64, intermediate_size=96, num_attention_heads=4, num_key_value_heads=2,
                         num_hidden_layers=2, vocab_size=101, rope_theta=10000.0, rms_norm_eps=1e-5,
                         max_position_embeddings=128, attention_bias=False, mlp_bias=False)
    hf = tr.LlamaModel(cfg).eval()
    sd = {k[len("model."):]: v for k, v in ours.state_dict().items() if k.startswith("model.")}
    hf.load_state_dict(sd, strict=True)
    ids = next(calibration_batches(s.vocab, 2, 12, 2, seed=8))
    with torch.no_grad():
        a = ours(ids)
        b = hf(input_ids=ids).last_hidden_state
    assert torch.allclose(a, b, atol=1e-5, rtol=1e-5), float((a - b).abs().max())


# --- structural tests of the reference's model classes (Llama*Tests.cs), on this calibration model
def _tiny():
    from llmcompressorsharp_b200.calibration import LlamaShape

    return LlamaShape(hidden=16, intermediate=24, heads=4, kv_heads=2, layers=2, vocab=50)


def test_rmsnorm_kats():  # LlamaRMSNormTests.cs:17-56
    from llmcompressorsharp_b200.calibration import RMSNorm

    n = RMSNorm(8, 1e-6, torch.float32, "cpu")
    x = torch.randn(2, 4, 8, generator=torch.Generator().manual_seed(3))
    y = n(x)
    assert list(y.shape) == [2, 4, 8]
    assert abs(float(y.pow(2).mean(-1).mean()) - 1.0) < 1e-3  # unit weight -> unit RMS rows
    assert float(n(torch.zeros(1, 8)).abs().max()) < 1e-5
    assert [list(p.shape) for p in n.parameters()] == [[8]]


def test_rotary_kats():  # LlamaRotaryEmbeddingTests.cs:17-70
    from llmcompressorsharp_b200.calibration import LlamaForCalibration, _rope

    m = LlamaForCalibration(_tiny(), dtype=torch.float32)
    cos, sin = m.rope_tables(4, torch.float32)
    q = torch.randn(1, 2, 4, 4, generator=torch.Generator().manual_seed(4))
    r = _rope(q, cos, sin)
    assert list(r.shape) == [1, 2, 4, 4]
    # each (i, i + half) pair is rotated, so its magnitude is kept
    half = q.shape[-1] // 2
    mag = lambda t: t[..., :half].pow(2) + t[..., half:].pow(2)  # noqa: E731
    assert torch.allclose(mag(r), mag(q), atol=1e-3)
    assert float((r[:, :, 0] - q[:, :, 0]).abs().max()) < 1e-5  # position 0 is the identity


def test_model_submodules_kats():  # LlamaMLPTests.cs, LlamaAttentionTests.cs, LlamaDecoderLayerTests.cs
    from llmcompressorsharp_b200.calibration import LlamaForCalibration

    m = LlamaForCalibration(_tiny(), dtype=torch.float32)
    layer = m.model.layers[0]
    mlp = {n for n, _ in layer.mlp.named_parameters()}
    assert mlp == {"gate_proj.weight", "up_proj.weight", "down_proj.weight"}  # three Linear layers, no bias
    attn = {n for n, _ in layer.self_attn.named_parameters()}
    assert attn == {"q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight"}
    names = {n for n, _ in layer.named_children()}
    assert {"input_layernorm", "self_attn", "post_attention_layernorm", "mlp"} <= names
    top = {n for n, _ in m.model.named_children()}
    assert {"embed_tokens", "layers", "norm"} <= top  # no lm_head: calibration stops at the decoder
    cos, sin = m.rope_tables(5, torch.float32)
    x = torch.randn(2, 5, 16, generator=torch.Generator().manual_seed(5))
    y = layer(x, cos, sin)
    assert list(y.shape) == [2, 5, 16] and float((y - x).abs().max()) > 1e-5  # residual adds something
