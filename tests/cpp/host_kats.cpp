// Known-answer tests of the C++ host mirror (include/llmc_b200.hpp), one per case of the
// reference's xUnit tests (tests/LLMCompressorSharp.Tests/...), run on the GPU through the C ABI.
// Exit status 0 when every test passes.  Build and run: tests/test_cpp_host.py.
#include <cmath>
#include <cstdio>
#include <functional>
#include <string>
#include <vector>

#include "llmc_b200.hpp"

using namespace llmcs;

namespace {

struct Failure {
    std::string what;
};

void Assert(bool ok, const std::string& what) {
    if (!ok) throw Failure{what};
}

void Near(float got, float want, float tol, const std::string& what) {
    Assert(std::fabs(got - want) <= tol, what + ": got " + std::to_string(got) + ", want " + std::to_string(want));
}

template <typename E, typename F>
void Throws(F f, const std::string& what) {
    try {
        f();
    } catch (const E&) {
        return;
    } catch (const std::exception& e) {
        throw Failure{what + ": wrong exception: " + e.what()};
    }
    throw Failure{what + ": nothing thrown"};
}

std::vector<std::pair<std::string, std::function<void(Context&)>>> tests() {
    std::vector<std::pair<std::string, std::function<void(Context&)>>> t;

    // ---- HessianAccumulatorTests.cs
    t.push_back({"HessianAccumulator.InitialIsZero", [](Context& c) {  // :16-25
                     HessianAccumulator acc(c, 4);
                     Assert(acc.SampleCount() == 0, "sample count");
                     for (float v : acc.GetHessian().ToHost()) Assert(v == 0.f, "zero H");
                 }});
    t.push_back({"HessianAccumulator.OneBatchIsOuterProduct", [](Context& c) {  // :27-43
                     HessianAccumulator acc(c, 3);
                     acc.Update(DeviceTensor::FromHost({1, 2, 3}, {1, 3}));
                     Assert(acc.SampleCount() == 1, "sample count");
                     const std::vector<float> want = {1, 2, 3, 2, 4, 6, 3, 6, 9};
                     Assert(acc.GetHessian().ToHost() == want, "H = x^T x");
                 }});
    t.push_back({"HessianAccumulator.BatchesAreAdditive", [](Context& c) {  // :45-58
                     HessianAccumulator acc(c, 2);
                     acc.Update(DeviceTensor::FromHost({1, 0}, {1, 2}));
                     acc.Update(DeviceTensor::FromHost({0, 1}, {1, 2}));
                     Assert(acc.SampleCount() == 2, "sample count");
                     Assert(acc.GetHessian().ToHost() == std::vector<float>({1, 0, 0, 1}), "H");
                 }});
    t.push_back({"HessianAccumulator.HighRankInputIsFlattened", [](Context& c) {  // :60-83
                     HessianAccumulator acc(c, 2);
                     acc.Update(DeviceTensor::FromHost({1, 0, 0, 1, 1, 1, 1, 0, 0, 1, 1, 1}, {2, 3, 2}));
                     Assert(acc.SampleCount() == 6, "sample count");
                     Assert(acc.GetHessian().ToHost() == std::vector<float>({4, 2, 2, 4}), "H");
                 }});
    t.push_back({"HessianAccumulator.WrongLastDimThrows", [](Context& c) {  // :85-92
                     HessianAccumulator acc(c, 3);
                     Throws<ArgumentException>([&] { acc.Update(DeviceTensor::FromHost({1, 2}, {1, 2})); }, "last dim");
                 }});
    t.push_back({"HessianAccumulator.HalfInputAccumulatesInFloat32", [](Context& c) {  // :94-103
                     HessianAccumulator acc(c, 2);
                     acc.Update(DeviceTensor::FromHost({1, 2}, {1, 2}, DType::Float16));
                     const DeviceTensor h = acc.GetHessian();
                     Assert(h.dtype() == DType::Float32, "fp32 H");
                     Assert(h.ToHost() == std::vector<float>({1, 2, 2, 4}), "H");
                 }});
    t.push_back({"HessianAccumulator.Reset", [](Context& c) {  // :105-116
                     HessianAccumulator acc(c, 2);
                     acc.Update(DeviceTensor::FromHost({1, 2}, {1, 2}));
                     acc.Reset();
                     Assert(acc.SampleCount() == 0, "sample count");
                     for (float v : acc.GetHessian().ToHost()) Assert(v == 0.f, "zero H");
                 }});
    t.push_back({"HessianAccumulator.NonPositiveInFeaturesThrows", [](Context& c) {  // :118-123
                     Throws<ArgumentOutOfRangeException>([&] { HessianAccumulator acc(c, 0); }, "inFeatures 0");
                 }});

    // ---- HessianInverseSolverTests.cs
    t.push_back({"HessianInverseSolver.Identity", [](Context& c) {  // :17-27
                     std::vector<float> eye(16, 0.f);
                     for (int i = 0; i < 4; i++) eye[5 * i] = 1.f;
                     const auto h = HessianInverseSolver::Compute(c, DeviceTensor::FromHost(eye, {4, 4}), 0.f).ToHost();
                     for (int i = 0; i < 16; i++) Near(h[i], eye[i], 1e-5f, "I^-1");
                 }});
    t.push_back({"HessianInverseSolver.ScaledIdentity", [](Context& c) {  // :29-39
                     std::vector<float> two(9, 0.f);
                     for (int i = 0; i < 3; i++) two[4 * i] = 2.f;
                     const auto h = HessianInverseSolver::Compute(c, DeviceTensor::FromHost(two, {3, 3}), 0.f).ToHost();
                     for (int i = 0; i < 9; i++) Near(h[i], i % 4 == 0 ? 0.5f : 0.f, 1e-5f, "(2I)^-1");
                 }});
    t.push_back({"HessianInverseSolver.RankDeficientDampedIsFinite", [](Context& c) {  // :41-51
                     const auto h = HessianInverseSolver::Compute(c, DeviceTensor::FromHost({1, 1, 1, 1}, {2, 2}), 0.01f).ToHost();
                     for (float v : h) Assert(std::isfinite(v), "finite");
                 }});
    t.push_back({"HessianInverseSolver.ZeroMatrixFallsBackToPinvZero", [](Context& c) {  // :85-91 (pinv(0) = 0)
                     const auto h = HessianInverseSolver::Compute(c, DeviceTensor::FromHost(std::vector<float>(25, 0.f), {5, 5}),
                                                                   0.01f).ToHost();
                     for (float v : h) Assert(v == 0.f, "zero");
                 }});
    t.push_back({"HessianInverseSolver.SingularFallsBackToPinv", [](Context& c) {  // :85-91
                     // diag(2, 0, 4, 0) has no Cholesky factor; pinv keeps the non-zero eigenvalues.
                     std::vector<float> h(16, 0.f);
                     h[0] = 2.f;
                     h[10] = 4.f;
                     const auto p = HessianInverseSolver::Compute(c, DeviceTensor::FromHost(h, {4, 4}), 0.f).ToHost();
                     for (int i = 0; i < 16; i++)
                         Near(p[i], i == 0 ? 0.5f : (i == 10 ? 0.25f : 0.f), 1e-6f, "pinv(diag(2, 0, 4, 0))");
                 }});
    t.push_back({"HessianInverseSolver.NonSquareThrows", [](Context& c) {  // :72-78
                     Throws<ArgumentException>(
                         [&] { HessianInverseSolver::Compute(c, DeviceTensor::FromHost(std::vector<float>(12, 1.f), {3, 4}), 0.01f); },
                         "square");
                 }});

    // ---- MinMaxObserverTests.cs
    t.push_back({"MinMaxObserver.AccumulatesAsymmetric", [](Context& c) {  // :22-42
                     MinMaxObserver obs(c);
                     for (const auto& b : {std::vector<float>{-2, 0, 3}, std::vector<float>{-5, 1, 2}, std::vector<float>{-1, 7, 0}})
                         obs.Update(DeviceTensor::FromHost(b, {3}));
                     const auto p = obs.GetQuantParams(8, false);
                     Near(p.Scale[0], 12.f / 255.f, 1e-5f, "scale");
                     Assert(p.ZeroPoint[0] == 106, "zero-point 106");
                 }});
    t.push_back({"MinMaxObserver.Symmetric", [](Context& c) {  // :44-58
                     MinMaxObserver obs(c);
                     obs.Update(DeviceTensor::FromHost({-3, 0, 5}, {3}));
                     const auto p = obs.GetQuantParams(8, true);
                     Near(p.Scale[0], 5.f / 127.f, 1e-5f, "scale");
                     Assert(p.ZeroPoint[0] == 0, "zero-point");
                 }});
    t.push_back({"MinMaxObserver.Reset", [](Context& c) {  // :60-74
                     MinMaxObserver obs(c);
                     obs.Update(DeviceTensor::FromHost({-10, 10}, {2}));
                     obs.Reset();
                     obs.Update(DeviceTensor::FromHost({-1, 1}, {2}));
                     Near(obs.GetQuantParams(8, true).Scale[0], 1.f / 127.f, 1e-5f, "scale");
                 }});
    t.push_back({"MinMaxObserver.NoSamplesThrows", [](Context& c) {  // :76-83
                     MinMaxObserver obs(c);
                     Throws<InvalidOperationException>([&] { obs.GetQuantParams(8, true); }, "no samples");
                 }});
    t.push_back({"MinMaxObserver.AllZerosGiveScaleOne", [](Context& c) {  // :85-95
                     MinMaxObserver obs(c);
                     obs.Update(DeviceTensor::FromHost({0, 0, 0}, {3}));
                     const auto p = obs.GetQuantParams(8, true);
                     Assert(p.Scale[0] == 1.f && p.ZeroPoint[0] == 0, "(1, 0)");
                 }});
    t.push_back({"Observer.BitsOutOfRangeThrow", [](Context& c) {  // Observer.cs:53-56
                     MinMaxObserver obs(c);
                     obs.Update(DeviceTensor::FromHost({-1, 1}, {2}));
                     Throws<ArgumentOutOfRangeException>([&] { obs.GetQuantParams(1, true); }, "bits 1");
                 }});

    // ---- PerChannelMinMaxObserverTests.cs
    t.push_back({"PerChannelMinMaxObserver.OneScalePerRow", [](Context& c) {  // :118-143
                     PerChannelMinMaxObserver obs(c, 0);
                     obs.Update(DeviceTensor::FromHost({-2, 0, 4, -10, 5, 10}, {2, 3}));
                     const auto p = obs.GetQuantParams(8, true);
                     Assert(p.Scale.size() == 2, "two scales");
                     Near(p.Scale[0], 4.f / 127.f, 1e-5f, "scale 0");
                     Near(p.Scale[1], 10.f / 127.f, 1e-5f, "scale 1");
                 }});
    t.push_back({"PerChannelMinMaxObserver.Accumulates", [](Context& c) {  // :145-171
                     PerChannelMinMaxObserver obs(c, 0);
                     obs.Update(DeviceTensor::FromHost({-1, 2, -3, 5}, {2, 2}));
                     obs.Update(DeviceTensor::FromHost({-5, 1, -2, 8}, {2, 2}));
                     const auto p = obs.GetQuantParams(8, true);
                     Near(p.Scale[0], 5.f / 127.f, 1e-5f, "scale 0");
                     Near(p.Scale[1], 8.f / 127.f, 1e-5f, "scale 1");
                 }});
    t.push_back({"PerChannelMinMaxObserver.ResetAndErrors", [](Context& c) {  // :173-219
                     PerChannelMinMaxObserver obs(c, 0);
                     Throws<InvalidOperationException>([&] { obs.GetQuantParams(8, true); }, "no samples");
                     obs.Update(DeviceTensor::FromHost({-10, 10, -20, 20}, {2, 2}));
                     obs.Reset();
                     obs.Update(DeviceTensor::FromHost({-1, 1, -2, 2}, {2, 2}));
                     const auto p = obs.GetQuantParams(8, true);
                     Near(p.Scale[0], 1.f / 127.f, 1e-5f, "scale 0");
                     Near(p.Scale[1], 2.f / 127.f, 1e-5f, "scale 1");
                     PerChannelMinMaxObserver bad(c, 5);
                     Throws<ArgumentOutOfRangeException>([&] { bad.Update(DeviceTensor::FromHost({1, 1, 1, 1}, {2, 2})); },
                                                         "axis 5");
                 }});

    // ---- FakeQuantizeFunctionTests.cs
    t.push_back({"FakeQuantize.Symmetric8", [](Context& c) {  // :16-30
                     const auto y = FakeQuantize::Apply(c, DeviceTensor::FromHost({-127.4f, -127.6f, 0.4f, 0.6f, 127.4f, 127.6f}, {6}),
                                                        1.f, 0, 8, true).ToHost();
                     Assert(y == std::vector<float>({-127, -127, 0, 1, 127, 127}), "grid");
                 }});
    t.push_back({"FakeQuantize.Symmetric4Scale", [](Context& c) {  // :32-43
                     const auto y = FakeQuantize::Apply(c, DeviceTensor::FromHost({-3.6f, 0.f, 3.6f}, {3}), 0.5f, 0, 4, true).ToHost();
                     Assert(y == std::vector<float>({-3.5f, 0.f, 3.5f}), "grid");
                 }});
    t.push_back({"FakeQuantize.AsymmetricZeroPoint", [](Context& c) {  // :60-73
                     const auto y = FakeQuantize::Apply(c, DeviceTensor::FromHost({-8.f, 0.f, 7.f}, {3}), 1.f, 8, 4, false).ToHost();
                     Assert(y == std::vector<float>({-8.f, 0.f, 7.f}), "grid");
                 }});
    t.push_back({"FakeQuantize.InvalidBitsThrow", [](Context& c) {  // :75-81
                     Throws<ArgumentOutOfRangeException>(
                         [&] { FakeQuantize::Apply(c, DeviceTensor::FromHost({1.f, 2.f}, {2}), 1.f, 0, 1, true); }, "bits 1");
                 }});

    // ---- Int4PackedTensorTests.cs
    t.push_back({"Int4PackedTensor.ClampsSymmetric", [](Context& c) {  // :16-31
                     auto p = Int4PackedTensor::FromFloat(c, DeviceTensor::FromHost({-8.5f, -7.f, 0.f, 7.f, 9.f}, {5}), 1.f, 0, true);
                     Assert(p.Dequantize().ToHost() == std::vector<float>({-7, -7, 0, 7, 7}), "clamped");
                 }});
    t.push_back({"Int4PackedTensor.HalvesStorage", [](Context& c) {  // :33-41
                     auto p = Int4PackedTensor::FromFloat(c, DeviceTensor::FromHost({1, 2, 3, 4, 5, 6, 7, 8}, {8}), 1.f, 0, true);
                     Assert(p.PackedBytes().size() == 4, "4 bytes");
                 }});
    t.push_back({"Int4PackedTensor.RoundTrip", [](Context& c) {  // :43-59
                     const std::vector<float> vals = {-7, -3, 0, 4, 7, -2};
                     auto p = Int4PackedTensor::FromFloat(c, DeviceTensor::FromHost(vals, {6}), 1.f, 0, true);
                     auto r = Int4PackedTensor::FromPackedBytes(c, p.PackedBytes(), 6, 1.f, 0, true);
                     Assert(r.Dequantize().ToHost() == vals, "round trip");
                 }});
    t.push_back({"Int4PackedTensor.NibbleOrder", [](Context& c) {  // Int4PackedTensor.cs:52-64
                     auto p = Int4PackedTensor::FromFloat(c, DeviceTensor::FromHost({1.f, 2.f, -1.f}, {3}), 1.f, 0, true);
                     Assert(p.PackedBytes() == std::vector<uint8_t>({0x12, 0xF0}), "even index in the high nibble");
                     Throws<ArgumentException>([&] { Int4PackedTensor::FromPackedBytes(c, {0x12}, 3, 1.f, 0, true); }, "length");
                 }});

    // ---- GptqBlockQuantizerTests.cs / GPTQModifierTests.cs
    t.push_back({"GptqBlockQuantizer.ZeroWeightStaysZero", [](Context& c) {  // GptqBlockQuantizerTests.cs:18-30
                     std::vector<float> eye(16, 0.f);
                     for (int i = 0; i < 4; i++) eye[5 * i] = 1.f;
                     GPTQConfig cfg;
                     cfg.NumBits = 8;
                     cfg.Strategy = QuantizationStrategy::PerTensor;
                     const auto q = GptqBlockQuantizer::Quantize(c, DeviceTensor::FromHost(std::vector<float>(8, 0.f), {2, 4}),
                                                                 DeviceTensor::FromHost(eye, {4, 4}), cfg).ToHost();
                     for (float v : q) Near(v, 0.f, 1e-6f, "zero");
                 }});
    t.push_back({"GptqBlockQuantizer.SixteenBitIsNearIdentity", [](Context& c) {  // :115-138
                     GPTQConfig cfg;
                     cfg.NumBits = 16;
                     cfg.Strategy = QuantizationStrategy::PerTensor;
                     cfg.BlockSize = 1;
                     const auto q = GptqBlockQuantizer::Quantize(c, DeviceTensor::FromHost({1, 2, 3, 4}, {2, 2}),
                                                                 DeviceTensor::FromHost({1, 0, 0, 1}, {2, 2}), cfg).ToHost();
                     const std::vector<float> w = {1, 2, 3, 4};
                     for (int i = 0; i < 4; i++) Near(q[i], w[i], 0.01f, "identity");
                 }});
    t.push_back({"GptqBlockQuantizer.ActOrderThrows", [](Context& c) {  // GPTQModifierTests.cs:130-141
                     GPTQConfig cfg;
                     cfg.ActOrder = true;
                     Throws<NotSupportedException>(
                         [&] {
                             GptqBlockQuantizer::Quantize(c, DeviceTensor::FromHost({1, 1, 1, 1}, {2, 2}),
                                                          DeviceTensor::FromHost({1, 0, 0, 1}, {2, 2}), cfg);
                         },
                         "ActOrder");
                 }});
    // ---- extensions of the mirror (no reference test): context controls, per-token codes, AWQ's
    // apply step, activation order, the allocation-free observer
    t.push_back({"Context.ControlsAndLaunchCount", [](Context& c) {
                     const int64_t n0 = c.LaunchCount();
                     c.SetSmLimit(16);
                     c.SetWaitLimit(-1);
                     c.SetDeferredErrors(true);
                     HessianAccumulator acc(c, 8);
                     acc.Update(DeviceTensor::FromHost(std::vector<float>(64, 1.f), {8, 8}));
                     c.Synchronize();
                     c.SetDeferredErrors(false);
                     c.SetSmLimit(0);
                     Assert(c.LaunchCount() > n0, "launch count grows");
                     Assert(acc.GetHessian().ToHost()[0] == 8.f, "H[0][0]");
                 }});
    t.push_back({"PerTokenQuantizer.SymmetricInt8", [](Context& c) {
                     // row 0 absmax 127 -> scale 1; row 1 absmax 254 -> scale 2
                     auto r = PerTokenQuantizer::Quantize(c, DeviceTensor::FromHost({127, -64, 3, 0, 254, -127, 7, 1}, {2, 4}));
                     Near(r.Scales[0], 1.f, 0.f, "scale 0");
                     Near(r.Scales[1], 2.f, 0.f, "scale 1");
                     Assert((int8_t)r.Codes[0] == 127 && (int8_t)r.Codes[1] == -64 && (int8_t)r.Codes[2] == 3, "row 0");
                     // 254 / 2 = 127; -127 / 2 = -63.5 -> -64 (half to even); 7 / 2 = 3.5 -> 4; 1 / 2 -> 0
                     Assert((int8_t)r.Codes[4] == 127 && (int8_t)r.Codes[5] == -64 && (int8_t)r.Codes[6] == 4 &&
                                (int8_t)r.Codes[7] == 0,
                            "row 1");
                 }});
    t.push_back({"ScaleApply.BalanceTimesSmoothOver", [](Context& c) {
                     auto s = DeviceTensor::FromHost({2, 4}, {2});
                     auto smooth = DeviceTensor::FromHost({8, 8}, {2});
                     auto balance = DeviceTensor::FromHost({1, 1, 0.5f, 0.25f}, {2, 2});
                     ScaleApply::Apply(c, s, &smooth, balance);
                     const std::vector<float> sm = smooth.ToHost(), bal = balance.ToHost();
                     Assert(sm[0] == 4.f && sm[1] == 2.f, "smooth / s");
                     Assert(bal[0] == 2.f && bal[1] == 4.f && bal[2] == 1.f && bal[3] == 1.f, "balance * s");
                 }});
    t.push_back({"ActOrder.DecreasingDiagonal", [](Context& c) {
                     auto h = DeviceTensor::FromHost({1, 0, 0, 0, 3, 0, 0, 0, 2}, {3, 3});
                     const std::vector<int32_t> want = {1, 2, 0};
                     Assert(ActOrder::Permutation(c, h) == want, "order by diag(H) descending");
                 }});
    t.push_back({"NoAllocObserver.MinMax", [](Context& c) {
                     DeviceTensor mn({1}, DType::Float32), mx({1}, DType::Float32);
                     NoAllocObserver::MinMax(c, DeviceTensor::FromHost({-3, 5, 2, 0.5f}, {2, 2}), mn, mx);
                     Assert(mn.ToHost()[0] == -3.f && mx.ToHost()[0] == 5.f, "min / max");
                     NoAllocObserver::MinMax(c, DeviceTensor::FromHost({-1, 9}, {1, 2}), mn, mx, true);
                     Assert(mn.ToHost()[0] == -3.f && mx.ToHost()[0] == 9.f, "running min / max");
                 }});
    // ---- TargetMatcher / ModifierBase / GPTQModifierTests.cs / RtnModifierTests.cs / EndToEndRecipeTests.cs
    t.push_back({"TargetMatcher.GlobsAndIgnore", [](Context&) {  // TargetMatcher.cs:22-86
                     Assert(TargetMatcher::Matches("model.layers.0.q_proj.weight", {"model.*"}, {}), "glob");
                     Assert(!TargetMatcher::Matches("model.lm_head.weight", {"model.*"}, {"model.lm_head.*"}), "ignore wins");
                     Assert(TargetMatcher::Matches("anything", {}, {}), "no targets match all");
                     Assert(TargetMatcher::Matches("a.b", {"a.b"}, {}) && !TargetMatcher::Matches("a.bc", {"a.b"}, {}), "exact");
                     Assert(TargetMatcher::Matches("x.q_proj.weight", {"*q_proj*"}, {}), "two stars");
                     Assert(!TargetMatcher::Matches("x", {""}, {}), "empty pattern");
                 }});
    t.push_back({"ModifierBase.LifecycleOrder", [](Context& c) {  // ModifierBase.cs:47-180
                     CompressionState st;
                     st.NamedWeights.emplace_back("w", DeviceTensor::FromHost({1, 2}, {2}));
                     RtnModifier m(c, RtnConfig{8, true, QuantizationStrategy::PerTensor});
                     Throws<ModifierLifecycleException>([&] { m.OnStart(st); }, "start before initialize");
                     m.Initialize(st);
                     Throws<ModifierLifecycleException>([&] { m.Initialize(st); }, "initialize twice");
                     Throws<ModifierLifecycleException>([&] { m.OnEnd(st); }, "end before start");
                     m.OnStart(st);
                     m.OnEnd(st);
                     Throws<ModifierLifecycleException>([&] { m.OnBatch(st); }, "batch after end");
                     m.Finalize(st);
                     Throws<ModifierLifecycleException>([&] { m.Finalize(st); }, "finalize twice");
                 }});
    t.push_back({"RtnModifier.TargetsAndIgnore", [](Context& c) {  // EndToEndRecipeTests.cs:41-101 (its RTN stage)
                     CompressionState st;
                     st.NamedWeights.emplace_back("model.layer.0.weight", DeviceTensor::FromHost({1, 2, 3, 4, 5, 6, 7, 8}, {8}));
                     st.NamedWeights.emplace_back("model.lm_head.weight", DeviceTensor::FromHost({100, 200, 300}, {3}));
                     RtnModifier m(c, RtnConfig{8, true, QuantizationStrategy::PerTensor}, {"model.*"}, {"model.lm_head.*"});
                     m.Initialize(st);
                     m.OnStart(st);
                     m.OnEnd(st);
                     m.Finalize(st);
                     Assert(st.Weight("model.lm_head.weight").ToHost() == std::vector<float>({100, 200, 300}), "ignored");
                     const auto q = st.Weight("model.layer.0.weight").ToHost();
                     const float scale = 8.f / 127.f;  // Observer.cs:60-64, symmetric int8
                     for (int i = 0; i < 8; i++) {
                         const float want = std::nearbyint((float)(i + 1) / scale) * scale;
                         Near(q[i], want, 1e-6f, "fake-quantised value " + std::to_string(i));
                     }
                 }});
    t.push_back({"RtnModifier.PerTokenThrows", [](Context& c) {  // RtnModifier.cs:69-70
                     CompressionState st;
                     st.NamedWeights.emplace_back("w", DeviceTensor::FromHost({1, 2}, {1, 2}));
                     RtnModifier m(c, RtnConfig{8, true, QuantizationStrategy::PerToken});
                     m.Initialize(st);
                     m.OnStart(st);
                     Throws<NotSupportedException>([&] { m.OnEnd(st); }, "PerToken");
                 }});
    t.push_back({"GPTQModifier.RequiresNamedModules", [](Context& c) {  // GPTQModifierTests.cs:108-122
                     CompressionState st;
                     st.NamedWeights.emplace_back("linear.weight", DeviceTensor::FromHost(std::vector<float>(12, 0.5f), {3, 4}));
                     GPTQModifier m(c, GPTQConfig{});
                     Assert(m.Name() == "GPTQ", "name");
                     m.Initialize(st);
                     Throws<InvalidOperationException>([&] { m.OnStart(st); }, "NamedModules");
                 }});
    t.push_back({"GPTQModifier.ActOrderThrows", [](Context& c) {  // GPTQModifierTests.cs:124-136
                     CompressionState st;
                     GPTQConfig cfg;
                     cfg.ActOrder = true;
                     GPTQModifier m(c, cfg);
                     Throws<NotSupportedException>([&] { m.Initialize(st); }, "ActOrder");
                 }});
    t.push_back({"GPTQModifier.NoBatchesIsRtn", [](Context& c) {  // GPTQModifierTests.cs:89-106: H = 0
                     const std::vector<float> w = {0.3f, -1.2f, 0.05f, 2.0f, -0.7f, 0.9f, 1.13f, -0.4f, 0.6f, -2.2f, 0.15f, 0.8f};
                     CompressionState st;
                     st.NamedWeights.emplace_back("linear.weight", DeviceTensor::FromHost(w, {3, 4}));
                     st.NamedModules = {"linear"};
                     st.HasNamedModules = true;
                     GPTQConfig cfg;
                     cfg.NumBits = 8;
                     cfg.Strategy = QuantizationStrategy::PerTensor;
                     cfg.BlockSize = 4;
                     GPTQModifier m(c, cfg);
                     m.Initialize(st);
                     m.OnStart(st);
                     m.OnEnd(st);
                     m.Finalize(st);
                     const auto got = st.Weight("linear.weight").ToHost();
                     // pinv(0) = 0, U = Hinv = 0, every pivot skipped: the RTN fake-quantisation.
                     const auto want = Rtn::Quantize(c, DeviceTensor::FromHost(w, {3, 4}), RtnConfig{8, true, QuantizationStrategy::PerTensor})
                                           .Dequantized.ToHost();
                     for (size_t i = 0; i < w.size(); i++) Near(got[i], want[i], 0.f, "RTN value " + std::to_string(i));
                 }});
    t.push_back({"GPTQModifier.ObservedLayerAt16BitIsClose", [](Context& c) {  // GPTQModifierTests.cs:58-87
                     std::vector<float> w(12), x(24);
                     for (int i = 0; i < 12; i++) w[i] = std::sin(0.7f * i + 0.3f);
                     for (int i = 0; i < 24; i++) x[i] = std::cos(1.3f * i) + 0.1f * i;
                     CompressionState st;
                     st.NamedWeights.emplace_back("linear.weight", DeviceTensor::FromHost(w, {3, 4}));
                     st.NamedModules = {"linear"};
                     st.HasNamedModules = true;
                     GPTQConfig cfg;
                     cfg.NumBits = 16;
                     GPTQModifier m(c, cfg);
                     m.Initialize(st);
                     m.OnStart(st);
                     for (int b = 0; b < 3; b++) {
                         m.Observe("linear", DeviceTensor::FromHost(std::vector<float>(x.begin() + 8 * b, x.begin() + 8 * b + 8), {2, 4}));
                         m.OnBatch(st);
                     }
                     m.OnEnd(st);
                     m.Finalize(st);
                     const auto got = st.Weight("linear.weight").ToHost();
                     for (int i = 0; i < 12; i++) Near(got[i], w[i], 1e-3f, "16-bit GPTQ value " + std::to_string(i));
                 }});
    t.push_back({"GPTQModifier.SingularHessianTakesPinv", [](Context& c) {  // HessianInverseSolver.cs:85-91
                     std::vector<float> w(32), x(64 * 8);
                     for (int i = 0; i < 32; i++) w[i] = 0.05f * std::sin(1.1f * i);
                     for (int i = 0; i < 64 * 8; i++) x[i] = (i % 8 == 3) ? 0.f : std::sin(0.37f * i) + std::cos(0.11f * i * i);
                     CompressionState st;
                     st.NamedWeights.emplace_back("fc.weight", DeviceTensor::FromHost(w, {4, 8}));
                     st.NamedModules = {"fc"};
                     st.HasNamedModules = true;
                     GPTQConfig cfg;
                     cfg.DampeningFrac = 0.f;  // no damping: the dead input channel 3 leaves H singular
                     GPTQModifier m(c, cfg);
                     m.Initialize(st);
                     m.OnStart(st);
                     m.Observe("fc", DeviceTensor::FromHost(x, {64, 8}));
                     m.OnEnd(st);
                     m.Finalize(st);
                     const auto got = st.Weight("fc.weight").ToHost();
                     // The reference's composition: Hinv = pinv(H) (HessianInverseSolver.Compute), then
                     // GptqBlockQuantizer.Quantize with its U = chol(Hinv)^T or U = Hinv.
                     HessianAccumulator acc(c, 8);
                     acc.Update(DeviceTensor::FromHost(x, {64, 8}));
                     auto hinv = HessianInverseSolver::Compute(c, acc.GetHessian(), 0.f);
                     const auto want = GptqBlockQuantizer::Quantize(c, DeviceTensor::FromHost(w, {4, 8}), hinv, cfg).ToHost();
                     for (int i = 0; i < 32; i++) {
                         Assert(std::isfinite(got[i]), "finite");
                         Near(got[i], want[i], 1e-6f, "value " + std::to_string(i));
                     }
                 }});
    t.push_back({"SmoothQuantModifier.OutputPreservedAndScaled", [](Context& c) {  // SmoothQuantModifierTests.cs:26-76
                     CompressionState st;
                     st.NamedWeights.emplace_back("norm.weight", DeviceTensor::FromHost({2, 4}, {2}));
                     st.NamedWeights.emplace_back("proj.weight", DeviceTensor::FromHost({1, 1, 1, 1}, {2, 2}));
                     const DeviceTensor act = DeviceTensor::FromHost({1, 4, -0.5f, -2}, {2, 2});
                     st.LayerActivations = {{"proj", &act}};
                     st.HasLayerActivations = true;
                     SmoothQuantConfig cfg;
                     cfg.SmoothingStrength = 0.5f;
                     cfg.Mappings = {{"norm.weight", "proj.weight", "proj"}};
                     SmoothQuantModifier m(c, cfg);
                     Assert(m.Name() == "SmoothQuant", "name");
                     m.Initialize(st);
                     m.OnStart(st);
                     m.OnBatch(st);
                     m.OnEnd(st);
                     m.Finalize(st);
                     const auto g = st.Weight("norm.weight").ToHost(), w = st.Weight("proj.weight").ToHost();
                     Near(g[0], 2.f, 1e-4f, "g0");
                     Near(g[1], 2.f, 1e-4f, "g1");
                     Near(w[0], 1.f, 1e-4f, "w00");
                     Near(w[1], 2.f, 1e-4f, "w01");
                     Near(w[2], 1.f, 1e-4f, "w10");
                     Near(w[3], 2.f, 1e-4f, "w11");
                 }});
    t.push_back({"SmoothQuantModifier.PreservesIdentity", [](Context& c) {  // SmoothQuantModifierTests.cs:78-123
                     const std::vector<float> g = {1, 2, 3}, w = {0.5f, 1, -1, 2, -0.5f, 0.25f}, x = {0.1f, 0.5f, -1, 0.2f, -0.3f, 0.7f};
                     std::vector<float> xg(6), yref(4, 0.f);
                     for (int r = 0; r < 2; r++)
                         for (int k = 0; k < 3; k++) xg[3 * r + k] = x[3 * r + k] * g[k];
                     for (int r = 0; r < 2; r++)
                         for (int o = 0; o < 2; o++)
                             for (int k = 0; k < 3; k++) yref[2 * r + o] += xg[3 * r + k] * w[3 * o + k];
                     CompressionState st;
                     st.NamedWeights.emplace_back("g.weight", DeviceTensor::FromHost(g, {3}));
                     st.NamedWeights.emplace_back("proj.weight", DeviceTensor::FromHost(w, {2, 3}));
                     const DeviceTensor act = DeviceTensor::FromHost(xg, {2, 3});
                     st.LayerActivations = {{"proj", &act}};
                     st.HasLayerActivations = true;
                     SmoothQuantConfig cfg;
                     cfg.Mappings = {{"g.weight", "proj.weight", "proj"}};
                     SmoothQuantModifier m(c, cfg);
                     m.Initialize(st);
                     m.OnStart(st);
                     m.OnBatch(st);
                     m.OnEnd(st);
                     m.Finalize(st);
                     const auto gn = st.Weight("g.weight").ToHost(), wn = st.Weight("proj.weight").ToHost();
                     for (int r = 0; r < 2; r++)
                         for (int o = 0; o < 2; o++) {
                             float y = 0.f;
                             for (int k = 0; k < 3; k++) y += x[3 * r + k] * gn[k] * wn[3 * o + k];
                             Near(y, yref[2 * r + o], 1e-4f, "y");
                         }
                 }});
    t.push_back({"SmoothQuantModifier.AlphaOutOfRangeThrows", [](Context& c) {  // SmoothQuantModifier.cs:25-31
                     SmoothQuantConfig cfg;
                     cfg.SmoothingStrength = 1.5f;
                     Throws<ArgumentOutOfRangeException>([&] { SmoothQuantModifier m(c, cfg); }, "alpha");
                 }});
    t.push_back({"SmoothQuantModifier.NoActivationThrows", [](Context& c) {  // SmoothQuantModifier.cs:118-127
                     CompressionState st;
                     st.NamedWeights.emplace_back("norm.weight", DeviceTensor::FromHost({2, 4}, {2}));
                     st.NamedWeights.emplace_back("proj.weight", DeviceTensor::FromHost({1, 1, 1, 1}, {2, 2}));
                     SmoothQuantConfig cfg;
                     cfg.Mappings = {{"norm.weight", "proj.weight", "proj"}};
                     SmoothQuantModifier m(c, cfg);
                     m.Initialize(st);
                     m.OnStart(st);
                     Throws<InvalidOperationException>([&] { m.OnEnd(st); }, "no activation");
                 }});
    t.push_back({"SparseGPTModifier.TwoFourMask", [](Context& c) {  // phase-4c-sparsegpt.md:1584-1656 (2:4)
                     std::vector<float> w(32), x(64 * 8);
                     for (int i = 0; i < 32; i++) w[i] = 0.05f * std::sin(1.7f * i + 0.2f);
                     for (int i = 0; i < 64 * 8; i++) x[i] = std::sin(0.37f * i) + std::cos(0.11f * i * i);
                     CompressionState st;
                     st.NamedWeights.emplace_back("fc.weight", DeviceTensor::FromHost(w, {4, 8}, DType::BFloat16));
                     st.NamedWeights.emplace_back("other.weight", DeviceTensor::FromHost(w, {4, 8}));
                     st.NamedModules = {"fc", "other"};
                     st.HasNamedModules = true;
                     SparseGPTConfig cfg;
                     cfg.MaskN = 2;
                     cfg.MaskM = 4;
                     SparseGPTModifier m(c, cfg);
                     Assert(m.Name() == "SparseGPT", "name");
                     m.Initialize(st);
                     m.OnStart(st);
                     m.Observe("fc", DeviceTensor::FromHost(x, {64, 8}));  // "other" sees no calibration rows
                     m.OnEnd(st);
                     m.Finalize(st);
                     Assert(st.Weight("fc.weight").dtype() == DType::BFloat16, "dtype kept");
                     const auto p = st.Weight("fc.weight").ToHost();
                     for (int r = 0; r < 4; r++)
                         for (int g = 0; g < 2; g++) {
                             int zeros = 0;
                             for (int k = 0; k < 4; k++) zeros += p[8 * r + 4 * g + k] == 0.f;
                             Assert(zeros >= 2, "2:4 group " + std::to_string(r) + "," + std::to_string(g));
                         }
                     Assert(st.Weight("other.weight").ToHost() == w, "no calibration rows: unchanged");
                 }});
    t.push_back({"AWQModifier.SearchesAndApplies", [](Context& c) {  // algorithm-mapping.md:214-249
                     const int n = 128, m = 4, rows = 16;
                     std::vector<float> w(m * n), g(n), x(rows * n);
                     for (int i = 0; i < m * n; i++) w[i] = 0.02f * std::sin(0.9f * i + 0.1f);
                     for (int i = 0; i < n; i++) g[i] = 1.f + 0.1f * std::cos(0.5f * i);
                     for (int i = 0; i < rows * n; i++) x[i] = std::sin(0.23f * i) * ((i % n) % 17 == 0 ? 20.f : 1.f);
                     CompressionState st;
                     st.NamedWeights.emplace_back("norm.weight", DeviceTensor::FromHost(g, {n}));
                     st.NamedWeights.emplace_back("proj.weight", DeviceTensor::FromHost(w, {m, n}));
                     const DeviceTensor act = DeviceTensor::FromHost(x, {rows, n});
                     st.LayerActivations = {{"proj", &act}};
                     st.HasLayerActivations = true;
                     AWQConfig cfg;
                     cfg.Mappings = {{"norm.weight", "proj.weight", "proj"}};
                     AWQModifier mod(c, cfg);
                     mod.Initialize(st);
                     mod.OnStart(st);
                     mod.OnBatch(st);
                     mod.OnEnd(st);
                     mod.Finalize(st);
                     Assert(mod.Chosen.size() == 1 && mod.Chosen[0].first == "proj.weight", "one mapping");
                     DeviceTensor amax({n}, DType::Float32);
                     SmoothQuant::UpdateActivationMax(c, act, amax, false);
                     const AwqResult want = AWQ::Search(c, DeviceTensor::FromHost(w, {m, n}), amax, 20, cfg.Quant);
                     Assert(mod.Chosen[0].second == want.BestK && want.BestK >= 1 && want.BestK <= 20, "grid point");
                     const auto gn = st.Weight("norm.weight").ToHost(), wn = st.Weight("proj.weight").ToHost();
                     for (int i = 0; i < n; i++) {
                         Near(gn[i], g[i] / want.BestScale[i], 1e-6f * std::fabs(g[i] / want.BestScale[i]) + 1e-30f, "smooth / s");
                         for (int r = 0; r < m; r++)
                             Near(wn[r * n + i], w[r * n + i] * want.BestScale[i],
                                  1e-6f * std::fabs(w[r * n + i] * want.BestScale[i]) + 1e-30f, "balance * s");
                     }
                 }});
    t.push_back({"CompressionSession.CompletesFailsAndRunsOnce", [](Context& c) {  // CompressionSession.cs
                     // GPTQ over two batches fed by the host's forward, then RTN of the other weight.
                     std::vector<float> w(12);
                     for (int i = 0; i < 12; i++) w[i] = std::sin(0.7f * i + 0.3f);
                     CompressionState st;
                     st.NamedWeights.emplace_back("linear.weight", DeviceTensor::FromHost(w, {3, 4}));
                     st.NamedWeights.emplace_back("head.weight", DeviceTensor::FromHost({1, 2, 3, 4, 5, 6, 7, 8}, {8}));
                     st.NamedModules = {"linear"};
                     st.HasNamedModules = true;
                     GPTQConfig gc;
                     gc.NumBits = 16;
                     GPTQModifier gptq(c, gc, {"linear.*"});
                     RtnModifier rtn(c, RtnConfig{8, true, QuantizationStrategy::PerTensor}, {"head.*"});
                     CompressionSession session({&gptq, &rtn});
                     int fed = 0;
                     const auto status = session.Run(st, 2, [&](CompressionState&, int b) {
                         std::vector<float> x(8);
                         for (int i = 0; i < 8; i++) x[i] = std::cos(1.3f * (i + 8 * b)) + 0.1f * i;
                         gptq.Observe("linear", DeviceTensor::FromHost(x, {2, 4}));
                         fed++;
                     });
                     Assert(status == SessionStatus::Completed && fed == 2, "completed");
                     const auto q = st.Weight("linear.weight").ToHost();
                     for (int i = 0; i < 12; i++) Near(q[i], w[i], 1e-3f, "16-bit GPTQ");
                     const auto h = st.Weight("head.weight").ToHost();
                     const float scale = 8.f / 127.f;
                     for (int i = 0; i < 8; i++) Near(h[i], std::nearbyint((float)(i + 1) / scale) * scale, 1e-6f, "RTN");
                     Throws<InvalidOperationException>([&] { session.Run(st, 0, nullptr); }, "run once");
                     // A modifier that throws: the session fails, keeps the exception, finalises.
                     CompressionState bad;
                     bad.NamedWeights.emplace_back("linear.weight", DeviceTensor::FromHost(w, {3, 4}));
                     GPTQModifier needsModules(c, GPTQConfig{});
                     CompressionSession s2({&needsModules});
                     Assert(s2.Run(bad, 1, nullptr) == SessionStatus::Failed, "failed");
                     Throws<InvalidOperationException>([&] { std::rethrow_exception(s2.Failure()); }, "failure kept");
                 }});
    return t;
}

}  // namespace

int main() {
    Context ctx(0);
    int failed = 0, passed = 0;
    for (auto& [name, fn] : tests()) {
        try {
            fn(ctx);
            passed++;
        } catch (const Failure& f) {
            failed++;
            std::printf("FAIL %s: %s\n", name.c_str(), f.what.c_str());
        } catch (const std::exception& e) {
            failed++;
            std::printf("FAIL %s: unexpected exception: %s\n", name.c_str(), e.what());
        }
    }
    std::printf("%d passed, %d failed\n", passed, failed);
    return failed == 0 ? 0 : 1;
}
