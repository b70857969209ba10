// Host logic of the C++ mirror (include/llmc_b200.hpp) that needs no GPU: target matching
// (TargetMatcher.cs:22-86), the modifier lifecycle checks (ModifierBase.cs:47-180), the session's
// order, failure capture and finalisation (CompressionSession.cs), and the status -> exception
// mapping of the C ABI.  Exit status 0 when every test passes.  Build and run:
// tests/test_cpp_host.py.
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

// A modifier that records its hooks; `throwAt` names the hook that throws.
class Recorder : public ModifierBase {
   public:
    Recorder(std::string name, std::vector<std::string>* log, std::string throwAt = "")
        : ModifierBase(std::move(name), {}, {}), log_(log), throw_(std::move(throwAt)) {}

   protected:
    void OnInitialize(CompressionState&) override { Hook("init"); }
    void OnStartCore(CompressionState&) override { Hook("start"); }
    void OnBatchCore(CompressionState&) override { Hook("batch"); }
    void OnEndCore(CompressionState&) override { Hook("end"); }
    void OnFinalizeCore(CompressionState&) override { Hook("final"); }

   private:
    void Hook(const std::string& h) {
        log_->push_back(Name() + ":" + h);
        if (h == throw_) throw InvalidOperationException(Name() + " failed at " + h);
    }
    std::vector<std::string>* log_;
    std::string throw_;
};

std::vector<std::pair<std::string, std::function<void()>>> tests() {
    std::vector<std::pair<std::string, std::function<void()>>> t;
    t.push_back({"TargetMatcher.Patterns", [] {  // TargetMatcherTests / TargetMatcher.cs:22-86
                     Assert(TargetMatcher::Matches("model.layers.0.q_proj.weight", {"model.*"}, {}), "prefix glob");
                     Assert(TargetMatcher::Matches("model.layers.0.q_proj.weight", {"*q_proj*"}, {}), "infix glob");
                     Assert(TargetMatcher::Matches("a/b.c", {"a*c"}, {}), "star crosses separators");
                     Assert(!TargetMatcher::Matches("model.lm_head.weight", {"model.*"}, {"*lm_head*"}), "ignore wins");
                     Assert(TargetMatcher::Matches("x", {}, {}), "no targets");
                     Assert(!TargetMatcher::Matches("x", {}, {"x"}), "ignored with no targets");
                     Assert(TargetMatcher::Matches("abc", {"abc"}, {}) && !TargetMatcher::Matches("abcd", {"abc"}, {}), "exact");
                     Assert(!TargetMatcher::Matches("abc", {""}, {}), "empty pattern");
                     Assert(TargetMatcher::Matches("aaa", {"a*a*a"}, {}) && !TargetMatcher::Matches("aa", {"a*a*a"}, {}),
                            "backtracking");
                     Assert(TargetMatcher::Matches("", {"*"}, {}), "star matches empty");
                 }});
    t.push_back({"ModifierBase.Lifecycle", [] {  // ModifierBase.cs:47-180
                     std::vector<std::string> log;
                     Recorder m("m", &log);
                     CompressionState st;
                     Throws<ModifierLifecycleException>([&] { m.OnStart(st); }, "start before init");
                     Throws<ModifierLifecycleException>([&] { m.Finalize(st); }, "finalize before init");
                     m.Initialize(st);
                     Throws<ModifierLifecycleException>([&] { m.Initialize(st); }, "init twice");
                     Throws<ModifierLifecycleException>([&] { m.OnBatch(st); }, "batch before start");
                     m.OnStart(st);
                     Throws<ModifierLifecycleException>([&] { m.OnStart(st); }, "start twice");
                     m.OnBatch(st);
                     m.OnEnd(st);
                     Throws<ModifierLifecycleException>([&] { m.OnEnd(st); }, "end twice");
                     Throws<ModifierLifecycleException>([&] { m.OnBatch(st); }, "batch after end");
                     m.Finalize(st);
                     Throws<ModifierLifecycleException>([&] { m.Finalize(st); }, "finalize twice");
                     Assert(log == std::vector<std::string>({"m:init", "m:start", "m:batch", "m:end", "m:final"}), "hooks");
                 }});
    t.push_back({"CompressionSession.Order", [] {  // CompressionSession.cs
                     std::vector<std::string> log;
                     Recorder a("a", &log), b("b", &log);
                     CompressionState st;
                     CompressionSession s({&a, &b});
                     int fed = 0;
                     Assert(s.Status() == SessionStatus::NotStarted, "not started");
                     Assert(s.Run(st, 2, [&](CompressionState&, int i) { Assert(i == fed++, "batch index"); }) ==
                                SessionStatus::Completed,
                            "completed");
                     Assert(log == std::vector<std::string>({"a:init", "b:init", "a:start", "b:start", "a:batch", "b:batch",
                                                             "a:batch", "b:batch", "a:end", "b:end", "a:final", "b:final"}),
                            "order");
                     Throws<InvalidOperationException>([&] { s.Run(st, 0, nullptr); }, "run once");
                 }});
    t.push_back({"CompressionSession.FailureKeptAndInitializedFinalized", [] {  // CompressionSession.cs
                     std::vector<std::string> log;
                     Recorder a("a", &log), b("b", &log, "init"), c("c", &log);
                     CompressionState st;
                     CompressionSession s({&a, &b, &c});
                     Assert(s.Run(st, 1, nullptr) == SessionStatus::Failed, "failed");
                     Throws<InvalidOperationException>([&] { std::rethrow_exception(s.Failure()); }, "failure kept");
                     // b threw inside Initialize after being marked initialised; c never was.
                     Assert(log == std::vector<std::string>({"a:init", "b:init", "a:final"}), "only a finalised");
                     Throws<ArgumentNullException>([&] { CompressionSession bad({nullptr}); }, "null modifier");
                 }});
    t.push_back({"Check.StatusToException", [] {  // the shim's mapping of the C ABI's statuses
                     Throws<ArgumentException>([] { Check(LLMC_ERR_SHAPE); }, "shape");
                     Throws<ArgumentException>([] { Check(LLMC_ERR_INVALID_ARG); }, "invalid arg");
                     Throws<ArgumentOutOfRangeException>([] { Check(LLMC_ERR_OUT_OF_RANGE); }, "out of range");
                     Throws<NotSupportedException>([] { Check(LLMC_ERR_UNSUPPORTED); }, "unsupported");
                     Throws<InvalidOperationException>([] { Check(LLMC_ERR_NO_SAMPLES); }, "no samples");
                     try {
                         Check(LLMC_ERR_NOT_PD);
                         throw Failure{"NOT_PD: nothing thrown"};
                     } catch (const LlmcException& e) {
                         Assert(e.status == LLMC_ERR_NOT_PD, "NOT_PD status kept");
                     }
                     Check(LLMC_OK);
                 }});
    t.push_back({"Configs.DefaultsAndCLayout", [] {  // GPTQConfig.cs:22-59, GPTQConfigTests.cs:16-56
                     GPTQConfig g;
                     Assert(g.NumBits == 4 && g.Symmetric && g.Strategy == QuantizationStrategy::PerChannel &&
                                g.ChannelAxis == 0 && g.BlockSize == 128 && !g.ActOrder,
                            "GPTQ defaults");
                     Assert(g.DampeningFrac > 0.0099f && g.DampeningFrac < 0.0101f, "damp 0.01");
                     g.NumBits = 99;  // no validation in the config itself
                     g.BlockSize = 64;
                     g.Strategy = QuantizationStrategy::Group;
                     g.GroupSize = 32;
                     const llmc_qconfig c = g.ToC();
                     Assert(c.num_bits == 99 && c.block_size == 64 && c.strategy == LLMC_STRATEGY_GROUP && c.group_size == 32 &&
                                c.symmetric == 1 && c.act_order == 0,
                            "GPTQ to C");
                     const llmc_qconfig r = RtnConfig{8, false, QuantizationStrategy::PerTensor, 128}.ToC();
                     Assert(r.num_bits == 8 && r.symmetric == 0 && r.strategy == LLMC_STRATEGY_TENSOR, "RTN to C");
                     SmoothQuantConfig sq;
                     Assert(sq.SmoothingStrength == 0.5f && sq.Mappings.empty(), "SmoothQuant defaults");
                     AWQConfig aw;
                     Assert(aw.NGrid == 20 && aw.Quant.NumBits == 4 && !aw.Quant.Symmetric &&
                                aw.Quant.Strategy == QuantizationStrategy::Group && aw.Quant.GroupSize == 128,
                            "AWQ defaults");
                     SparseGPTConfig sp;
                     Assert(sp.Sparsity == 0.5f && sp.MaskN == 0 && sp.MaskM == 0 && sp.BlockSize == 128, "SparseGPT defaults");
                 }});
    return t;
}

}  // namespace

int main() {
    int failed = 0, passed = 0;
    for (auto& [name, fn] : tests()) {
        try {
            fn();
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
    return failed ? 1 : 0;
}
