/*
 * llmc_b200.hpp — C++ host mirror of LLMCompressorSharp's one-shot compression primitives,
 * over the C ABI of include/llmc_b200.h (header-only, C++17, links libllmc_b200 and cudart).
 *
 * The reference exposes these as C# classes on TorchSharp tensors
 * (src/LLMCompressorSharp.TorchExtensions, src/LLMCompressorSharp.Core/Algorithms/Gptq).  This
 * header keeps their names, argument meaning and exception behaviour:
 *   HessianAccumulator        HessianAccumulator.cs:16-99
 *   HessianInverseSolver      HessianInverseSolver.cs:44-108
 *   GptqBlockQuantizer        GptqBlockQuantizer.cs:71-274 (+ GPTQConfig, Configs/GPTQConfig.cs:22-59)
 *   MinMaxObserver            MinMaxObserver.cs:14-71
 *   PerChannelMinMaxObserver  PerChannelMinMaxObserver.cs:15-112
 *   FakeQuantize              FakeQuantize.cs:22-38
 *   Int4PackedTensor          Int4PackedTensor.cs:47-161
 *   TargetMatcher, ModifierBase, CompressionState (Core/Modifiers, Core/Compression)
 *   GPTQModifier              GPTQModifier.cs:28-155
 *   RtnModifier               RtnModifier.cs:44-122
 *   SmoothQuantModifier       SmoothQuantModifier.cs:15-182
 *   SparseGPTModifier, AWQModifier (the reference's plans: phase-4c-sparsegpt.md,
 *                             algorithm-mapping.md:214-249)
 *   CompressionSession        CompressionSession.cs
 * Tensors are DeviceTensor: a device buffer owned by the host code (the role TorchSharp's
 * CUDA tensors play for the C# primitives), row-major, float32 / bfloat16 / float16.
 * Exceptions mirror .NET's: ArgumentNullException, ArgumentException,
 * ArgumentOutOfRangeException, NotSupportedException, InvalidOperationException; CUDA and
 * timeout failures raise LlmcException.
 */
#ifndef LLMC_B200_HPP
#define LLMC_B200_HPP

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <functional>
#include <stdexcept>
#include <string>
#include <utility>
#include <limits>
#include <memory>
#include <vector>

#include "llmc_b200.h"

namespace llmcs {

// ---- exceptions ------------------------------------------------------------------------------
struct LlmcException : std::runtime_error {
    llmc_status status;
    LlmcException(llmc_status st, const std::string& m) : std::runtime_error(m), status(st) {}
};
struct ArgumentException : std::invalid_argument {
    explicit ArgumentException(const std::string& m) : std::invalid_argument(m) {}
};
struct ArgumentNullException : ArgumentException {
    explicit ArgumentNullException(const std::string& m) : ArgumentException(m) {}
};
struct ArgumentOutOfRangeException : ArgumentException {
    explicit ArgumentOutOfRangeException(const std::string& m) : ArgumentException(m) {}
};
struct NotSupportedException : std::logic_error {
    explicit NotSupportedException(const std::string& m) : std::logic_error(m) {}
};
struct InvalidOperationException : std::logic_error {
    explicit InvalidOperationException(const std::string& m) : std::logic_error(m) {}
};

// Maps a status of the C ABI (and the calling thread's message) to the reference's exception.
inline void Check(llmc_status st) {
    if (st == LLMC_OK) return;
    const char* e = llmc_last_error();
    const std::string m = e ? e : "llmc error";
    switch (st) {
        case LLMC_ERR_INVALID_ARG:
            if (m.find("must not be null") != std::string::npos) throw ArgumentNullException(m);
            throw ArgumentException(m);
        case LLMC_ERR_SHAPE: throw ArgumentException(m);
        case LLMC_ERR_OUT_OF_RANGE: throw ArgumentOutOfRangeException(m);
        case LLMC_ERR_UNSUPPORTED: throw NotSupportedException(m);
        case LLMC_ERR_NO_SAMPLES: throw InvalidOperationException(m);
        default: throw LlmcException(st, m);
    }
}

inline void CheckCuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw LlmcException(LLMC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// ---- device context ---------------------------------------------------------------------------
class Context {
   public:
    explicit Context(int device = 0) {
        Check(llmc_init(device, &ctx_));
        device_ = device;
    }
    ~Context() {
        if (ctx_) llmc_destroy(ctx_);
    }
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;
    llmc_ctx* get() const { return ctx_; }
    int device() const { return device_; }
    // Waits for the context's stream and raises its first deferred device error.
    void Synchronize() const { Check(llmc_sync(ctx_)); }
    // Extensions (no reference counterpart): the stream the context's work is ordered on, an SM
    // cap for its persistent grids (0: the whole GPU), the tries of a bounded device wait
    // (negative: the default), device-side "not positive definite" decisions reported by
    // Synchronize, and the number of kernels it has launched.
    void SetStream(cudaStream_t stream) { Check(llmc_set_stream(ctx_, (void*)stream)); }
    void SetSmLimit(int sms) { Check(llmc_set_sm_limit(ctx_, sms)); }
    void SetWaitLimit(int64_t tries) { Check(llmc_set_wait_limit(ctx_, tries)); }
    void SetDeferredErrors(bool on) { Check(llmc_set_deferred_errors(ctx_, on ? 1 : 0)); }
    int64_t LaunchCount() const {
        int64_t n = 0;
        Check(llmc_launch_count(ctx_, &n));
        return n;
    }

   private:
    llmc_ctx* ctx_ = nullptr;
    int device_ = 0;
};

// ---- tensors ---------------------------------------------------------------------------------
enum class DType : int32_t { Float32 = LLMC_DTYPE_F32, BFloat16 = LLMC_DTYPE_BF16, Float16 = LLMC_DTYPE_F16 };

inline size_t ElementSize(DType t) { return t == DType::Float32 ? 4 : 2; }

class DeviceTensor {
   public:
    DeviceTensor() = default;
    DeviceTensor(std::vector<int64_t> shape, DType dtype) : shape_(std::move(shape)), dtype_(dtype) {
        if (bytes()) CheckCuda(cudaMalloc(&data_, bytes()), "cudaMalloc");
    }
    // Host values converted to `dtype` (round to nearest even).
    static DeviceTensor FromHost(const std::vector<float>& values, std::vector<int64_t> shape, DType dtype = DType::Float32) {
        DeviceTensor t(std::move(shape), dtype);
        if ((int64_t)values.size() != t.numel()) throw ArgumentException("value count does not match the shape");
        std::vector<unsigned char> raw(t.bytes());
        for (size_t i = 0; i < values.size(); i++) {
            if (dtype == DType::Float32) std::memcpy(&raw[4 * i], &values[i], 4);
            else if (dtype == DType::BFloat16) {
                const __nv_bfloat16 h = __float2bfloat16_rn(values[i]);
                std::memcpy(&raw[2 * i], &h, 2);
            } else {
                const __half h = __float2half_rn(values[i]);
                std::memcpy(&raw[2 * i], &h, 2);
            }
        }
        if (t.bytes()) CheckCuda(cudaMemcpy(t.data_, raw.data(), t.bytes(), cudaMemcpyHostToDevice), "cudaMemcpy");
        return t;
    }
    std::vector<float> ToHost() const {
        std::vector<unsigned char> raw(bytes());
        if (bytes()) CheckCuda(cudaMemcpy(raw.data(), data_, bytes(), cudaMemcpyDeviceToHost), "cudaMemcpy");
        std::vector<float> out((size_t)numel());
        for (size_t i = 0; i < out.size(); i++) {
            if (dtype_ == DType::Float32) std::memcpy(&out[i], &raw[4 * i], 4);
            else if (dtype_ == DType::BFloat16) {
                __nv_bfloat16 h;
                std::memcpy(&h, &raw[2 * i], 2);
                out[i] = __bfloat162float(h);
            } else {
                __half h;
                std::memcpy(&h, &raw[2 * i], 2);
                out[i] = __half2float(h);
            }
        }
        return out;
    }
    ~DeviceTensor() {
        if (data_) cudaFree(data_);
    }
    DeviceTensor(DeviceTensor&& o) noexcept { *this = std::move(o); }
    DeviceTensor& operator=(DeviceTensor&& o) noexcept {
        if (this != &o) {
            if (data_) cudaFree(data_);
            data_ = o.data_;
            shape_ = std::move(o.shape_);
            dtype_ = o.dtype_;
            o.data_ = nullptr;
        }
        return *this;
    }
    DeviceTensor(const DeviceTensor&) = delete;
    DeviceTensor& operator=(const DeviceTensor&) = delete;

    void* data() const { return data_; }
    DType dtype() const { return dtype_; }
    const std::vector<int64_t>& shape() const { return shape_; }
    int64_t dim() const { return (int64_t)shape_.size(); }
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t s : shape_) n *= s;
        return n;
    }
    int64_t last() const { return shape_.empty() ? 1 : shape_.back(); }
    size_t bytes() const { return (size_t)numel() * ElementSize(dtype_); }

   private:
    void* data_ = nullptr;
    std::vector<int64_t> shape_;
    DType dtype_ = DType::Float32;
};

// ---- HessianAccumulator ------------------------------------------------------------------------
class HessianAccumulator {
   public:
    HessianAccumulator(Context& ctx, int inFeatures) : ctx_(&ctx), d_(inFeatures) {
        Check(llmc_hessian_create(ctx.get(), inFeatures, &h_));
    }
    ~HessianAccumulator() {
        if (h_) llmc_hessian_destroy(h_);
    }
    HessianAccumulator(const HessianAccumulator&) = delete;
    HessianAccumulator& operator=(const HessianAccumulator&) = delete;

    // H += X^T X over x viewed as [-1, inFeatures] (HessianAccumulator.cs:47-67).
    void Update(const DeviceTensor& x) {
        if (x.dim() == 0 || x.last() != d_)
            throw ArgumentException("Input last dim (" + std::to_string(x.last()) + ") must equal inFeatures (" +
                                    std::to_string(d_) + ").");
        Check(llmc_hessian_update(h_, x.data(), (int32_t)x.dtype(), x.numel() / d_, d_));
    }
    DeviceTensor GetHessian() const {
        DeviceTensor out({d_, d_}, DType::Float32);
        Check(llmc_hessian_get(h_, static_cast<float*>(out.data())));
        return out;
    }
    void Reset() { Check(llmc_hessian_reset(h_)); }
    int64_t SampleCount() const {
        int64_t n = 0;
        Check(llmc_hessian_sample_count(h_, &n));
        return n;
    }
    int InFeatures() const { return d_; }
    // The accumulator's own fp32 [d, d] buffer (upper triangle authoritative), no copy.
    const float* Data() const {
        float* p = nullptr;
        Check(llmc_hessian_data(h_, &p));
        return p;
    }
    // Multi-GPU: sum the partial H and sample counts of a token-sharded calibration set over
    // an NCCL communicator (an ncclComm_t), on every rank or onto `root`.
    void AllReduce(void* ncclComm) { Check(llmc_hessian_allreduce(h_, ncclComm)); }
    void Reduce(void* ncclComm, int root) { Check(llmc_hessian_reduce(h_, ncclComm, root)); }

   private:
    Context* ctx_;
    int d_;
    llmc_hessian* h_ = nullptr;
};

// ---- HessianInverseSolver ----------------------------------------------------------------------
struct HessianInverseSolver {
    // Damped inverse L^-T L^-1 of H + damp * mean(diag H) * I (HessianInverseSolver.cs:44-92).
    static DeviceTensor Compute(Context& ctx, const DeviceTensor& hessian, float dampingFrac) {
        if (hessian.dim() != 2 || hessian.shape()[0] != hessian.shape()[1])
            throw ArgumentException("Hessian must be a square 2-D tensor.");
        if (hessian.dtype() != DType::Float32) throw ArgumentException("Hessian must be float32.");
        const int64_t d = hessian.shape()[0];
        DeviceTensor out({d, d}, DType::Float32);
        Check(llmc_chol_inverse(ctx.get(), static_cast<const float*>(hessian.data()), d, d, dampingFrac, 0,
                                static_cast<float*>(out.data()), d, 0));
        return out;
    }
};

// ---- GPTQ -------------------------------------------------------------------------------------
enum class QuantizationStrategy : int32_t {
    PerTensor = LLMC_STRATEGY_TENSOR,
    PerChannel = LLMC_STRATEGY_CHANNEL,
    PerToken = LLMC_STRATEGY_TOKEN,
    Group = LLMC_STRATEGY_GROUP,  // the group-size extension
};

// Defaults of GPTQConfig.cs:22-59, plus GroupSize for the group strategy.
struct GPTQConfig {
    int NumBits = 4;
    bool Symmetric = true;
    QuantizationStrategy Strategy = QuantizationStrategy::PerChannel;
    int ChannelAxis = 0;
    int BlockSize = 128;
    float DampeningFrac = 0.01f;
    bool ActOrder = false;
    int GroupSize = 128;

    llmc_qconfig ToC() const {
        llmc_qconfig c{};
        c.num_bits = NumBits;
        c.symmetric = Symmetric ? 1 : 0;
        c.strategy = (int32_t)Strategy;
        c.channel_axis = ChannelAxis;
        c.group_size = GroupSize;
        c.block_size = BlockSize;
        c.damp = DampeningFrac;
        c.act_order = ActOrder ? 1 : 0;
        return c;
    }
};

struct GptqBlockQuantizer {
    // The fp32 fake-quantised weight (GptqBlockQuantizer.cs:71-190): U = chol(Hinv)^T with the
    // U = Hinv fallback, then the column-block solve.
    static DeviceTensor Quantize(Context& ctx, const DeviceTensor& weight, const DeviceTensor& hinv,
                                 const GPTQConfig& config) {
        if (weight.dim() != 2) throw ArgumentException("weight must be 2-D");
        const int64_t m = weight.shape()[0], n = weight.shape()[1];
        if (hinv.dim() != 2 || hinv.shape()[0] != n || hinv.shape()[1] != n)
            throw ArgumentException("hinv must be [in_features, in_features]");
        const llmc_qconfig c = config.ToC();
        DeviceTensor u({n, n}, DType::Float32);
        Check(llmc_upper_factor(ctx.get(), static_cast<const float*>(hinv.data()), n, n, static_cast<float*>(u.data()), n));
        const int64_t per_row = config.Strategy == QuantizationStrategy::Group ? (n + config.GroupSize - 1) / config.GroupSize : 1;
        const int64_t nparams = config.Strategy == QuantizationStrategy::PerTensor ? 1 : m * per_row;
        DeviceTensor scales({nparams}, DType::Float32), zps({nparams}, DType::Float32);  // int32 payload, 4-byte slots
        DeviceTensor out({m, n}, DType::Float32);
        Check(llmc_gptq_quantize(ctx.get(), weight.data(), (int32_t)weight.dtype(), m, n, n,
                                 static_cast<const float*>(u.data()), n, &c, static_cast<float*>(out.data()), n, nullptr,
                                 static_cast<float*>(scales.data()), static_cast<int32_t*>(zps.data())));
        return out;
    }
};

// ---- observers ----------------------------------------------------------------------------------
// Host copy of QuantizationParameters (QuantizationParameters.cs:21-25).
struct QuantizationParameters {
    std::vector<float> Scale;
    std::vector<int64_t> ZeroPoint;
    QuantizationStrategy Strategy;
};

namespace detail {
inline QuantizationParameters Affine(Context& ctx, const DeviceTensor& mins, const DeviceTensor& maxs, int64_t count,
                                     int numBits, bool symmetric, QuantizationStrategy st) {
    DeviceTensor s({count}, DType::Float32), z({count}, DType::Float32);
    Check(llmc_affine_params(ctx.get(), static_cast<const float*>(mins.data()), static_cast<const float*>(maxs.data()),
                             count, numBits, symmetric ? 1 : 0, static_cast<float*>(s.data()),
                             static_cast<int32_t*>(z.data())));
    QuantizationParameters p{s.ToHost(), {}, st};
    std::vector<int32_t> zi((size_t)count);
    CheckCuda(cudaMemcpy(zi.data(), z.data(), (size_t)count * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    p.ZeroPoint.assign(zi.begin(), zi.end());
    return p;
}
}  // namespace detail

class MinMaxObserver {
   public:
    explicit MinMaxObserver(Context& ctx) : ctx_(&ctx), mn_({1}, DType::Float32), mx_({1}, DType::Float32) {}
    // Running global min / max (MinMaxObserver.cs:24-45): starts at +inf / -inf and folds each
    // batch in by the observer's strict-less rule, so a batch holding a NaN changes nothing.
    void Update(const DeviceTensor& x) {
        if (x.numel() == 0) return;
        if (!has_) {
            const float init[2] = {std::numeric_limits<float>::infinity(), -std::numeric_limits<float>::infinity()};
            CheckCuda(cudaMemcpy(mn_.data(), &init[0], 4, cudaMemcpyHostToDevice), "cudaMemcpy");
            CheckCuda(cudaMemcpy(mx_.data(), &init[1], 4, cudaMemcpyHostToDevice), "cudaMemcpy");
        }
        Check(llmc_observer_minmax(ctx_->get(), x.data(), (int32_t)x.dtype(), x.numel() / x.last(), x.last(), x.last(),
                                   LLMC_STRATEGY_TENSOR, x.last(), static_cast<float*>(mn_.data()),
                                   static_cast<float*>(mx_.data()), 1));
        has_ = true;
    }
    QuantizationParameters GetQuantParams(int numBits, bool symmetric) {
        if (!has_) throw InvalidOperationException("MinMaxObserver has no calibration samples; call Update first.");
        return detail::Affine(*ctx_, mn_, mx_, 1, numBits, symmetric, QuantizationStrategy::PerTensor);
    }
    void Reset() { has_ = false; }

   private:
    Context* ctx_;
    DeviceTensor mn_, mx_;
    bool has_ = false;
};

// MSEObserver (MSEObserver.cs:17-124): samples kept on the device; the grid search over the
// symmetric ranges +-absMax*i/G runs in llmc_observer_mse.
class MSEObserver {
   public:
    MSEObserver(Context& ctx, int gridPoints = 100) : ctx_(&ctx), grid_(gridPoints) {
        if (gridPoints < 2) throw ArgumentOutOfRangeException("gridPoints must be >= 2.");
    }
    void Update(const DeviceTensor& x) {
        DeviceTensor copy({x.numel()}, x.dtype());
        if (x.bytes()) CheckCuda(cudaMemcpy(copy.data(), x.data(), x.bytes(), cudaMemcpyDeviceToDevice), "cudaMemcpy");
        samples_.push_back(std::move(copy));
    }
    QuantizationParameters GetQuantParams(int numBits, bool symmetric) {
        if (samples_.empty())
            throw InvalidOperationException("MSEObserver has no calibration samples. Call Update before GetQuantParams.");
        const DeviceTensor* flat = &samples_[0];
        DeviceTensor joined;
        if (samples_.size() > 1) {
            int64_t n = 0;
            for (const auto& t : samples_) {
                if (t.dtype() != samples_[0].dtype()) throw ArgumentException("samples must share one dtype");
                n += t.numel();
            }
            joined = DeviceTensor({n}, samples_[0].dtype());
            size_t off = 0;
            for (const auto& t : samples_) {
                if (t.bytes())
                    CheckCuda(cudaMemcpy(static_cast<char*>(joined.data()) + off, t.data(), t.bytes(),
                                         cudaMemcpyDeviceToDevice), "cudaMemcpy");
                off += t.bytes();
            }
            flat = &joined;
        }
        float scale = 1.f;
        int32_t zp = 0;
        Check(llmc_observer_mse(ctx_->get(), flat->data(), (int32_t)flat->dtype(), flat->numel(), grid_, numBits,
                                symmetric ? 1 : 0, &scale, &zp, nullptr));
        return QuantizationParameters{{scale}, {(int64_t)zp}, QuantizationStrategy::PerTensor};
    }
    void Reset() { samples_.clear(); }

   private:
    Context* ctx_;
    int grid_;
    std::vector<DeviceTensor> samples_;
};

class PerChannelMinMaxObserver {
   public:
    explicit PerChannelMinMaxObserver(Context& ctx, int channelAxis = 0) : ctx_(&ctx), axis_(channelAxis) {}
    // Running per-channel min / max over a 2-D tensor (PerChannelMinMaxObserver.cs:38-76).
    void Update(const DeviceTensor& x) {
        if (axis_ < 0 || axis_ >= x.dim())
            throw ArgumentOutOfRangeException("channelAxis " + std::to_string(axis_) + " is out of range for a " +
                                              std::to_string(x.dim()) + "-D tensor");
        if (axis_ != 0 || x.dim() != 2) throw NotSupportedException("per-channel statistics of axis 0 of a 2-D tensor");
        const int64_t rows = x.shape()[0], cols = x.shape()[1];
        if (has_ && rows != channels_) throw ArgumentException("channel count changed between updates");
        if (!has_) {
            mn_ = DeviceTensor({rows}, DType::Float32);
            mx_ = DeviceTensor({rows}, DType::Float32);
            channels_ = rows;
        }
        Check(llmc_observer_minmax(ctx_->get(), x.data(), (int32_t)x.dtype(), rows, cols, cols, LLMC_STRATEGY_CHANNEL, cols,
                                   static_cast<float*>(mn_.data()), static_cast<float*>(mx_.data()), has_ ? 1 : 0));
        has_ = true;
    }
    QuantizationParameters GetQuantParams(int numBits, bool symmetric) {
        if (!has_) throw InvalidOperationException("PerChannelMinMaxObserver has no calibration samples.");
        return detail::Affine(*ctx_, mn_, mx_, channels_, numBits, symmetric, QuantizationStrategy::PerChannel);
    }
    void Reset() { has_ = false; }

   private:
    Context* ctx_;
    int axis_;
    DeviceTensor mn_, mx_;
    int64_t channels_ = 0;
    bool has_ = false;
};

// ---- FakeQuantize / Int4PackedTensor --------------------------------------------------------------
struct FakeQuantize {
    // x.div(s).round().add(zp).clamp(qmin, qmax).sub(zp).mul(s) in x's dtype (FakeQuantize.cs:22-38).
    static DeviceTensor Apply(Context& ctx, const DeviceTensor& x, float scale, int64_t zeroPoint, int numBits,
                              bool symmetric) {
        DeviceTensor out(x.shape(), x.dtype());
        Check(llmc_fake_quantize(ctx.get(), x.data(), (int32_t)x.dtype(), x.numel(), scale, (int32_t)zeroPoint, numBits,
                                 symmetric ? 1 : 0, out.data(), nullptr));
        return out;
    }
};

class Int4PackedTensor {
   public:
    // Codes q = clamp(round(x / s) + zp) packed two per byte, even index in the high nibble
    // (Int4PackedTensor.cs:79-100, 47-69).
    static Int4PackedTensor FromFloat(Context& ctx, const DeviceTensor& x, float scale, int64_t zeroPoint, bool symmetric) {
        const int64_t n = x.numel();
        DeviceTensor codes({n}, DType::Float32);  // int32 payload
        Check(llmc_fake_quantize(ctx.get(), x.data(), (int32_t)x.dtype(), n, scale, (int32_t)zeroPoint, 4,
                                 symmetric ? 1 : 0, nullptr, static_cast<int32_t*>(codes.data())));
        Int4PackedTensor t(&ctx, n, scale, zeroPoint, symmetric);
        Check(llmc_int4_pack(ctx.get(), static_cast<const int32_t*>(codes.data()), n, (int32_t)zeroPoint,
                             static_cast<uint8_t*>(t.packed_.data())));
        return t;
    }
    // Int4PackedTensor.cs:111-149: (elementCount + 1) / 2 bytes, else ArgumentException.
    static Int4PackedTensor FromPackedBytes(Context& ctx, const std::vector<uint8_t>& packed, int64_t elementCount,
                                            float scale, int64_t zeroPoint, bool symmetric) {
        if ((int64_t)packed.size() != (elementCount + 1) / 2)
            throw ArgumentException("packed length must be (elementCount + 1) / 2");
        Int4PackedTensor t(&ctx, elementCount, scale, zeroPoint, symmetric);
        if (!packed.empty())
            CheckCuda(cudaMemcpy(t.packed_.data(), packed.data(), packed.size(), cudaMemcpyHostToDevice), "cudaMemcpy");
        return t;
    }
    std::vector<uint8_t> PackedBytes() const {
        std::vector<uint8_t> b((size_t)((n_ + 1) / 2));
        if (!b.empty()) CheckCuda(cudaMemcpy(b.data(), packed_.data(), b.size(), cudaMemcpyDeviceToHost), "cudaMemcpy");
        return b;
    }
    int64_t ElementCount() const { return n_; }
    // stored nibble (sign-extended only when symmetric) * scale (Int4PackedTensor.cs:152-161).
    DeviceTensor Dequantize() const {
        DeviceTensor out({n_}, DType::Float32);
        Check(llmc_int4_unpack_dequant(ctx_->get(), static_cast<const uint8_t*>(packed_.data()), n_, scale_,
                                       (int32_t)zp_, sym_ ? 1 : 0, static_cast<float*>(out.data())));
        return out;
    }

   private:
    Int4PackedTensor(Context* ctx, int64_t n, float s, int64_t zp, bool sym)
        : ctx_(ctx), n_(n), scale_(s), zp_(zp), sym_(sym), packed_({((n + 1) / 2 + 1) / 2}, DType::Float16) {}
    Context* ctx_;
    int64_t n_;
    float scale_;
    int64_t zp_;
    bool sym_;
    DeviceTensor packed_;  // (n + 1) / 2 bytes (allocated as 2-byte elements)
};

// ---- raw device bytes (codes, masks) ------------------------------------------------------------
class DeviceBytes {
   public:
    explicit DeviceBytes(size_t n) : n_(n) {
        if (n_) CheckCuda(cudaMalloc(&data_, n_), "cudaMalloc");
    }
    ~DeviceBytes() {
        if (data_) cudaFree(data_);
    }
    DeviceBytes(const DeviceBytes&) = delete;
    DeviceBytes& operator=(const DeviceBytes&) = delete;
    void* data() const { return data_; }
    size_t size() const { return n_; }
    template <typename T>
    std::vector<T> ToHost() const {
        std::vector<T> out(n_ / sizeof(T));
        if (n_) CheckCuda(cudaMemcpy(out.data(), data_, out.size() * sizeof(T), cudaMemcpyDeviceToHost), "cudaMemcpy");
        return out;
    }

   private:
    void* data_ = nullptr;
    size_t n_;
};

// ---- RTN (RtnModifier.cs:44-122 for one weight) -----------------------------------------------
struct RtnConfig {
    int NumBits = 4;
    bool Symmetric = true;
    QuantizationStrategy Strategy = QuantizationStrategy::PerChannel;
    int GroupSize = 128;

    llmc_qconfig ToC() const {
        llmc_qconfig c{};
        c.num_bits = NumBits;
        c.symmetric = Symmetric ? 1 : 0;
        c.strategy = (int32_t)Strategy;
        c.group_size = GroupSize;
        c.block_size = 128;
        return c;
    }
};

struct RtnResult {
    DeviceTensor Dequantized;           // the weight's dtype, like the reference's replacement weight
    std::vector<uint8_t> Codes;         // bits <= 4: (q - zp) & 0xF, two per byte, even column high
    std::vector<float> Scales;          // TENSOR: 1, CHANNEL: m, GROUP: m * ceil(n / GroupSize)
    std::vector<int32_t> ZeroPoints;
};

struct Rtn {
    static RtnResult Quantize(Context& ctx, const DeviceTensor& weight, const RtnConfig& config) {
        if (weight.dim() != 2) throw ArgumentException("weight must be 2-D");
        const int64_t m = weight.shape()[0], n = weight.shape()[1];
        const llmc_qconfig c = config.ToC();
        const int64_t per_row =
            config.Strategy == QuantizationStrategy::Group ? (n + config.GroupSize - 1) / config.GroupSize : 1;
        const int64_t nparams = config.Strategy == QuantizationStrategy::PerTensor ? 1 : m * per_row;
        const int64_t row_bytes = config.NumBits <= 4 ? (n + 1) / 2 : n;
        DeviceBytes codes((size_t)(m * row_bytes)), scales((size_t)nparams * 4), zps((size_t)nparams * 4);
        RtnResult r{DeviceTensor(weight.shape(), weight.dtype()), {}, {}, {}};
        Check(llmc_rtn_quantize(ctx.get(), weight.data(), (int32_t)weight.dtype(), m, n, n, &c,
                                static_cast<uint8_t*>(codes.data()), static_cast<float*>(scales.data()),
                                static_cast<int32_t*>(zps.data()), r.Dequantized.data()));
        r.Codes = codes.ToHost<uint8_t>();
        r.Scales = scales.ToHost<float>();
        r.ZeroPoints = zps.ToHost<int32_t>();
        return r;
    }
};

// ---- SmoothQuant (SmoothQuantModifier.cs:71-182) -----------------------------------------------
struct SmoothQuant {
    // UpdateActivationMax: runningMax[cols] = max(runningMax, max over rows |x|) (accumulate = false
    // overwrites); x is [-1, cols].
    static void UpdateActivationMax(Context& ctx, const DeviceTensor& x, DeviceTensor& runningMax, bool accumulate) {
        const int64_t cols = x.last();
        if (runningMax.numel() != cols || runningMax.dtype() != DType::Float32)
            throw ArgumentException("running max must be fp32 [cols]");
        Check(llmc_act_absmax(ctx.get(), x.data(), (int32_t)x.dtype(), x.numel() / cols, cols, cols,
                              static_cast<float*>(runningMax.data()), accumulate ? 1 : 0));
    }
    // ApplyMapping: smooth /= s, balance *= s in place; returns s.
    static std::vector<float> ApplyMapping(Context& ctx, const DeviceTensor& actMax, DeviceTensor& smooth,
                                           DeviceTensor& balance, float alpha) {
        if (balance.dim() != 2 || smooth.dim() != 1 || smooth.numel() != balance.last() || actMax.numel() != balance.last())
            throw ArgumentException("smooth must be 1-D and balance 2-D with matching last dims");
        DeviceTensor s({balance.last()}, DType::Float32);
        Check(llmc_smooth_apply(ctx.get(), static_cast<const float*>(actMax.data()), smooth.data(),
                                (int32_t)smooth.dtype(), balance.data(), (int32_t)balance.dtype(), balance.shape()[0],
                                balance.last(), alpha, static_cast<float*>(s.data())));
        return s.ToHost();
    }
};

// ---- AWQ's apply step with a given scale (algorithm-mapping.md:243-248) -------------------------
struct ScaleApply {
    // smooth /= s (skipped when smooth is null), balance *= s, in the weights' dtypes.
    static void Apply(Context& ctx, const DeviceTensor& s, DeviceTensor* smooth, DeviceTensor& balance) {
        if (balance.dim() != 2 || s.numel() != balance.last() || s.dtype() != DType::Float32)
            throw ArgumentException("balance must be 2-D and s fp32 [balance's last dim]");
        Check(llmc_scale_apply(ctx.get(), static_cast<const float*>(s.data()), smooth ? smooth->data() : nullptr,
                               smooth ? (int32_t)smooth->dtype() : 0, balance.data(), (int32_t)balance.dtype(),
                               balance.shape()[0], balance.last()));
    }
};

// ---- per-token activation quantisation (extension: W8A8's activation side) ---------------------
struct PerTokenResult {
    std::vector<uint8_t> Codes;       // [tokens, hidden]; two's complement for a symmetric grid
    std::vector<float> Scales;        // [tokens]
    std::vector<int32_t> ZeroPoints;  // [tokens]
};

struct PerTokenQuantizer {
    // x [tokens, hidden] (any leading shape folded into tokens); one min-max observer a row.
    static PerTokenResult Quantize(Context& ctx, const DeviceTensor& x, int numBits = 8, bool symmetric = true) {
        const int64_t cols = x.last(), rows = x.numel() / cols;
        DeviceBytes codes((size_t)(rows * cols)), scales((size_t)rows * 4), zps((size_t)rows * 4);
        Check(llmc_act_quant_per_token(ctx.get(), x.data(), (int32_t)x.dtype(), rows, cols, cols, numBits,
                                       symmetric ? 1 : 0, static_cast<uint8_t*>(codes.data()), cols,
                                       static_cast<float*>(scales.data()), static_cast<int32_t*>(zps.data()), nullptr,
                                       cols));
        return PerTokenResult{codes.ToHost<uint8_t>(), scales.ToHost<float>(), zps.ToHost<int32_t>()};
    }
};

// ---- GPTQ activation order (extension: the reference rejects ActOrder) -------------------------
struct ActOrder {
    // Columns in decreasing diag(H) (stable, NaN first); H fp32 [d, d].
    static std::vector<int32_t> Permutation(Context& ctx, const DeviceTensor& hessian) {
        if (hessian.dim() != 2 || hessian.shape()[0] != hessian.shape()[1] || hessian.dtype() != DType::Float32)
            throw ArgumentException("Hessian must be a square fp32 2-D tensor");
        const int64_t d = hessian.shape()[0];
        DeviceBytes perm((size_t)d * 4);
        Check(llmc_gptq_act_order_perm(ctx.get(), static_cast<const float*>(hessian.data()), d, d,
                                       static_cast<int32_t*>(perm.data())));
        return perm.ToHost<int32_t>();
    }
};

// ---- per-tensor min/max without device allocation (no reference counterpart) -------------------
struct NoAllocObserver {
    // For callers that may not allocate device memory mid-run (a hook on a model's stream, a
    // host allocator with a fixed budget): writes min / max into the caller's fp32 [1] device
    // tensors (updating them with accumulate) and allocates nothing; rows <= 65,536; calls that
    // overlap on the GPU share one static buffer and race.
    static void MinMax(Context& ctx, const DeviceTensor& x, DeviceTensor& minOut, DeviceTensor& maxOut,
                       bool accumulate = false) {
        if (minOut.numel() != 1 || maxOut.numel() != 1 || minOut.dtype() != DType::Float32 ||
            maxOut.dtype() != DType::Float32)
            throw ArgumentException("min / max must be fp32 tensors of one element");
        const int64_t cols = x.last(), rows = x.numel() / cols;
        Check(llmc_observer_minmax_tensor_noalloc(ctx.get(), x.data(), (int32_t)x.dtype(), rows, cols, cols,
                                                  static_cast<float*>(minOut.data()),
                                                  static_cast<float*>(maxOut.data()), accumulate ? 1 : 0));
    }
};

// ---- SparseGPT (plan phase-4c-sparsegpt.md, in GPTQ's U-factor form) --------------------------
struct SparseGPTResult {
    DeviceTensor Pruned;            // fp32 [m, n]
    std::vector<uint8_t> Mask;      // 1 = kept
};

struct SparseGPT {
    // maskN:maskM = 0:0 for unstructured pruning at `sparsity`, e.g. 2:4 for the N:M structure.
    static SparseGPTResult Prune(Context& ctx, const DeviceTensor& weight, const DeviceTensor& upper, float sparsity,
                                 int maskN, int maskM, int blockSize = 128) {
        if (weight.dim() != 2) throw ArgumentException("weight must be 2-D");
        const int64_t m = weight.shape()[0], n = weight.shape()[1];
        llmc_qconfig c{};
        c.num_bits = 8;
        c.symmetric = 1;
        c.block_size = blockSize;
        c.sparsity = sparsity;
        c.mask_n = maskN;
        c.mask_m = maskM;
        SparseGPTResult r{DeviceTensor({m, n}, DType::Float32), {}};
        DeviceBytes mask((size_t)(m * n));
        Check(llmc_sparsegpt_prune(ctx.get(), weight.data(), (int32_t)weight.dtype(), m, n, n,
                                   static_cast<const float*>(upper.data()), n, &c, static_cast<float*>(r.Pruned.data()), n,
                                   static_cast<uint8_t*>(mask.data())));
        r.Mask = mask.ToHost<uint8_t>();
        return r;
    }
};

// ---- AWQ grid search (algorithm-mapping.md:214-249) --------------------------------------------
struct AwqResult {
    std::vector<float> BestScale;   // per input channel
    std::vector<double> Mse;        // per grid point
    int BestK = 0;                  // 1-based grid index
};

struct AWQ {
    static AwqResult Search(Context& ctx, const DeviceTensor& weight, const DeviceTensor& actMax, int nGrid,
                            const RtnConfig& quant) {
        if (weight.dim() != 2) throw ArgumentException("weight must be 2-D");
        const int64_t m = weight.shape()[0], n = weight.shape()[1];
        const llmc_qconfig c = quant.ToC();
        DeviceBytes s((size_t)n * 4), mse((size_t)nGrid * 8);
        AwqResult r;
        int32_t k = 0;
        Check(llmc_awq_search(ctx.get(), weight.data(), (int32_t)weight.dtype(), m, n, n,
                              static_cast<const float*>(actMax.data()), nGrid, &c, static_cast<float*>(s.data()),
                              static_cast<double*>(mse.data()), &k));
        r.BestScale = s.ToHost<float>();
        r.Mse = mse.ToHost<double>();
        r.BestK = k;
        return r;
    }
};

// ---- NCCL communicator for the Hessian collectives ---------------------------------------------
class NcclCommunicator {
   public:
    // Rank 0 makes the id and sends it to the other ranks by the host's own channel.
    static std::vector<uint8_t> UniqueId() {
        std::vector<uint8_t> id(LLMC_NCCL_UNIQUE_ID_BYTES);
        Check(llmc_nccl_unique_id(id.data(), (int64_t)id.size()));
        return id;
    }
    NcclCommunicator(Context& ctx, int world, int rank, const std::vector<uint8_t>& id) {
        Check(llmc_nccl_comm_init(ctx.get(), world, rank, id.data(), (int64_t)id.size(), &comm_));
    }
    ~NcclCommunicator() {
        if (comm_) llmc_nccl_comm_destroy(comm_);
    }
    NcclCommunicator(const NcclCommunicator&) = delete;
    NcclCommunicator& operator=(const NcclCommunicator&) = delete;
    void* get() const { return comm_; }

   private:
    void* comm_ = nullptr;
};

// ---- modifiers (Core/Modifiers, Core/Compression, Algorithms/Gptq, Algorithms/Rtn) ---------------
struct ModifierLifecycleException : InvalidOperationException {
    explicit ModifierLifecycleException(const std::string& m) : InvalidOperationException(m) {}
};

// TargetMatcher.cs:22-86: ignore patterns win; no targets matches every name; a pattern without
// '*' matches exactly, and '*' matches any run of characters (dots and slashes included).
struct TargetMatcher {
    static bool MatchesPattern(const std::string& name, const std::string& pattern) {
        if (pattern.empty()) return false;
        if (pattern.find('*') == std::string::npos) return name == pattern;
        // Glob match with backtracking to the last '*'.
        size_t n = 0, p = 0, star = std::string::npos, mark = 0;
        while (n < name.size()) {
            if (p < pattern.size() && pattern[p] == '*') {
                star = p++;
                mark = n;
            } else if (p < pattern.size() && pattern[p] == name[n]) {
                p++;
                n++;
            } else if (star != std::string::npos) {
                p = star + 1;
                n = ++mark;
            } else {
                return false;
            }
        }
        while (p < pattern.size() && pattern[p] == '*') p++;
        return p == pattern.size();
    }
    static bool Matches(const std::string& name, const std::vector<std::string>& targets,
                        const std::vector<std::string>& ignore) {
        for (const auto& pat : ignore)
            if (MatchesPattern(name, pat)) return false;
        if (targets.empty()) return true;
        for (const auto& pat : targets)
            if (MatchesPattern(name, pat)) return true;
        return false;
    }
};

// CompressionState.cs:17-65.  NamedWeights keep the host's insertion order, as the C# dictionary
// enumerates.  The C# NamedModules (modules the modifiers hook) become the layer names whose
// inputs the host feeds to the modifiers' Observe(layerName, x): the call the hook lambda makes
// (ActivationHookManager.cs:47-51).
struct CompressionState {
    std::vector<std::pair<std::string, DeviceTensor>> NamedWeights;
    std::vector<std::string> NamedModules;
    bool HasNamedModules = false;
    // CompressionState.LayerActivations: this batch's activations by key, owned by the host,
    // which keeps them alive across the OnBatch / OnEnd call that reads them.
    std::vector<std::pair<std::string, const DeviceTensor*>> LayerActivations;
    bool HasLayerActivations = false;

    const DeviceTensor* Activation(const std::string& key) const {
        for (const auto& kv : LayerActivations)
            if (kv.first == key) return kv.second;
        return nullptr;
    }
    DeviceTensor& Weight(const std::string& name) {
        for (auto& kv : NamedWeights)
            if (kv.first == name) return kv.second;
        throw ArgumentException("no weight named " + name);
    }
    bool HasModule(const std::string& layer) const {
        for (const auto& m : NamedModules)
            if (m == layer) return true;
        return false;
    }
};

// ModifierBase.cs:47-180: the lifecycle checks and the hooks a modifier implements.
class ModifierBase {
   public:
    ModifierBase(std::string name, std::vector<std::string> targets, std::vector<std::string> ignore)
        : name_(std::move(name)), targets_(std::move(targets)), ignore_(std::move(ignore)) {}
    virtual ~ModifierBase() = default;
    const std::string& Name() const { return name_; }

    void Initialize(CompressionState& state) {
        if (initialized_) throw ModifierLifecycleException("Modifier '" + name_ + "' was initialized twice.");
        initialized_ = true;
        OnInitialize(state);
    }
    void OnStart(CompressionState& state) {
        EnsureInitialized();
        if (started_) throw ModifierLifecycleException("Modifier '" + name_ + "' was started twice.");
        started_ = true;
        OnStartCore(state);
    }
    void OnBatch(CompressionState& state) {
        EnsureStarted();
        if (ended_) throw ModifierLifecycleException("Modifier '" + name_ + "' received a batch after OnEnd.");
        OnBatchCore(state);
    }
    void OnEnd(CompressionState& state) {
        EnsureStarted();
        if (ended_) throw ModifierLifecycleException("Modifier '" + name_ + "' was ended twice.");
        ended_ = true;
        OnEndCore(state);
    }
    void Finalize(CompressionState& state) {
        if (!initialized_) throw ModifierLifecycleException("Modifier '" + name_ + "' was finalized before being initialized.");
        if (finalized_) throw ModifierLifecycleException("Modifier '" + name_ + "' was finalized twice.");
        finalized_ = true;
        OnFinalizeCore(state);
    }

   protected:
    virtual void OnInitialize(CompressionState&) {}
    virtual void OnStartCore(CompressionState&) {}
    virtual void OnBatchCore(CompressionState&) {}
    virtual void OnEndCore(CompressionState&) = 0;
    virtual void OnFinalizeCore(CompressionState&) {}
    std::vector<std::string> TargetedNames(const CompressionState& state) const {
        std::vector<std::string> out;
        for (const auto& kv : state.NamedWeights)
            if (TargetMatcher::Matches(kv.first, targets_, ignore_)) out.push_back(kv.first);
        return out;
    }

   private:
    void EnsureInitialized() const {
        if (!initialized_) throw ModifierLifecycleException("Modifier '" + name_ + "' was used before Initialize.");
    }
    void EnsureStarted() const {
        EnsureInitialized();
        if (!started_) throw ModifierLifecycleException("Modifier '" + name_ + "' was used before OnStart.");
    }
    std::string name_;
    std::vector<std::string> targets_, ignore_;
    bool initialized_ = false, started_ = false, ended_ = false, finalized_ = false;
};

// GPTQModifier.cs:28-155: one accumulator per targeted weight whose layer the host observes;
// OnEnd factors every Hessian and replaces each weight by its fp32 fake-quantised solve.  The
// factorisations are enqueued with the context's errors deferred and checked once; a Hessian
// without a Cholesky factor is factored again synchronously, which takes the reference's pinv
// fallback (HessianInverseSolver.cs:85-91).
class GPTQModifier : public ModifierBase {
   public:
    GPTQModifier(Context& ctx, GPTQConfig config, std::vector<std::string> targets = {},
                 std::vector<std::string> ignore = {})
        : ModifierBase("GPTQ", std::move(targets), std::move(ignore)), ctx_(&ctx), cfg_(config) {}

    // The hook: x is the input of layer `layerName` ([..., inFeatures]).
    void Observe(const std::string& layerName, const DeviceTensor& x) {
        for (auto& a : acc_)
            if (a.first == layerName + ".weight" || a.first == layerName) a.second->Update(x);
    }

   protected:
    void OnInitialize(CompressionState&) override {
        if (cfg_.ActOrder)
            throw NotSupportedException("GPTQConfig.ActOrder=true is not yet implemented. Column reordering by Hessian "
                                        "diagonal is deferred to a future release.");
    }
    void OnStartCore(CompressionState& state) override {
        if (!state.HasNamedModules)
            throw InvalidOperationException("GPTQModifier requires CompressionState.NamedModules to be populated.");
        acc_.clear();
        for (const auto& name : TargetedNames(state)) {
            const std::string suffix = ".weight";
            const bool has = name.size() >= suffix.size() && name.compare(name.size() - suffix.size(), suffix.size(), suffix) == 0;
            const std::string layer = has ? name.substr(0, name.size() - suffix.size()) : name;
            if (!state.HasModule(layer)) continue;
            const DeviceTensor& w = state.Weight(name);
            acc_.emplace_back(name, std::make_unique<HessianAccumulator>(*ctx_, (int)w.last()));
        }
    }
    void OnEndCore(CompressionState& state) override {
        std::vector<DeviceTensor> us;
        for (auto& a : acc_) us.emplace_back(std::vector<int64_t>{a.second->InFeatures(), a.second->InFeatures()}, DType::Float32);
        auto factor_all = [&] {
            for (size_t i = 0; i < acc_.size(); i++) {
                const int64_t d = acc_[i].second->InFeatures();
                Check(llmc_chol_inverse(ctx_->get(), acc_[i].second->Data(), d, d, cfg_.DampeningFrac, 1,
                                        static_cast<float*>(us[i].data()), d, 1));
            }
        };
        ctx_->SetDeferredErrors(true);
        bool redo = false;
        try {
            factor_all();
            ctx_->Synchronize();
        } catch (const LlmcException& e) {
            if (e.status != LLMC_ERR_NOT_PD) {
                ctx_->SetDeferredErrors(false);
                throw;
            }
            redo = true;
        }
        ctx_->SetDeferredErrors(false);
        if (redo) factor_all();
        const llmc_qconfig c = cfg_.ToC();
        for (size_t i = 0; i < acc_.size(); i++) {
            DeviceTensor& w = state.Weight(acc_[i].first);
            const int64_t m = w.shape()[0], n = w.shape()[1];
            const int64_t per_row = cfg_.Strategy == QuantizationStrategy::Group ? (n + cfg_.GroupSize - 1) / cfg_.GroupSize : 1;
            const int64_t nparams = cfg_.Strategy == QuantizationStrategy::PerTensor ? 1 : m * per_row;
            DeviceTensor scales({nparams}, DType::Float32), zps({nparams}, DType::Float32);
            DeviceTensor out({m, n}, DType::Float32);
            Check(llmc_gptq_quantize(ctx_->get(), w.data(), (int32_t)w.dtype(), m, n, n,
                                     static_cast<const float*>(us[i].data()), n, &c, static_cast<float*>(out.data()), n,
                                     nullptr, static_cast<float*>(scales.data()), static_cast<int32_t*>(zps.data())));
            w = std::move(out);
        }
    }
    void OnFinalizeCore(CompressionState&) override { acc_.clear(); }

   private:
    Context* ctx_;
    GPTQConfig cfg_;
    std::vector<std::pair<std::string, std::unique_ptr<HessianAccumulator>>> acc_;
};

// RtnModifier.cs:44-122: each targeted weight replaced by its fake-quantised value in its dtype.
// Any rank: per tensor the weight is one [1, numel] row; per channel (axis 0) it is
// [shape[0], numel / shape[0]], one channel a row; the group extension needs a 2-D weight.
class RtnModifier : public ModifierBase {
   public:
    RtnModifier(Context& ctx, RtnConfig config, std::vector<std::string> targets = {},
                std::vector<std::string> ignore = {})
        : ModifierBase("RTN", std::move(targets), std::move(ignore)), ctx_(&ctx), cfg_(config) {}

   protected:
    void OnEndCore(CompressionState& state) override {
        for (const auto& name : TargetedNames(state)) {
            if (cfg_.Strategy == QuantizationStrategy::PerToken)  // RtnModifier.cs:69-70
                throw NotSupportedException("PerToken strategy applies to activations, not weights.");
            DeviceTensor& w = state.Weight(name);
            const int64_t numel = w.numel();
            if (numel == 0) continue;
            int64_t m = 1, n = numel;
            if (cfg_.Strategy == QuantizationStrategy::PerChannel) {
                m = w.dim() == 0 ? 1 : w.shape()[0];
                n = numel / m;
            } else if (cfg_.Strategy == QuantizationStrategy::Group) {
                if (w.dim() != 2) throw ArgumentException("the group strategy needs a 2-D weight");
                m = w.shape()[0];
                n = w.shape()[1];
            }
            const llmc_qconfig c = cfg_.ToC();
            const int64_t per_row =
                cfg_.Strategy == QuantizationStrategy::Group ? (n + cfg_.GroupSize - 1) / cfg_.GroupSize : 1;
            const int64_t nparams = cfg_.Strategy == QuantizationStrategy::PerTensor ? 1 : m * per_row;
            const int64_t row_bytes = cfg_.NumBits <= 4 ? (n + 1) / 2 : n;
            DeviceBytes codes((size_t)(m * row_bytes)), scales((size_t)nparams * 4), zps((size_t)nparams * 4);
            DeviceTensor deq(w.shape(), w.dtype());
            Check(llmc_rtn_quantize(ctx_->get(), w.data(), (int32_t)w.dtype(), m, n, n, &c,
                                    static_cast<uint8_t*>(codes.data()), static_cast<float*>(scales.data()),
                                    static_cast<int32_t*>(zps.data()), deq.data()));
            w = std::move(deq);
        }
    }

   private:
    Context* ctx_;
    RtnConfig cfg_;
};

// SmoothQuantModifier.cs:15-182 with SmoothQuantConfig / SmoothQuantMapping
// (Configs/SmoothQuantConfig.cs): per mapping, the running per-channel |x| max of the activation
// key over the batches, then smooth /= s and balance *= s in the weights' dtypes.  The running
// maxima stay on the device (llmc_act_absmax folds each batch in).
struct SmoothQuantMapping {
    std::string SmoothWeight, BalanceWeight, ActivationKey;
};
struct SmoothQuantConfig {
    float SmoothingStrength = 0.5f;
    std::vector<SmoothQuantMapping> Mappings;
    std::vector<std::string> Targets, Ignore;
};

class SmoothQuantModifier : public ModifierBase {
   public:
    SmoothQuantModifier(Context& ctx, SmoothQuantConfig config)
        : ModifierBase("SmoothQuant", config.Targets, config.Ignore), ctx_(&ctx), cfg_(std::move(config)) {
        if (cfg_.SmoothingStrength < 0.f || cfg_.SmoothingStrength > 1.f)
            throw ArgumentOutOfRangeException("SmoothingStrength (alpha) must be in [0, 1].");
    }

   protected:
    void OnInitialize(CompressionState&) override { running_.clear(); }
    void OnBatchCore(CompressionState& state) override {
        if (!state.HasLayerActivations) return;
        for (const auto& mp : cfg_.Mappings)
            if (const DeviceTensor* x = state.Activation(mp.ActivationKey)) Update(mp.ActivationKey, *x);
    }
    void OnEndCore(CompressionState& state) override {
        for (const auto& mp : cfg_.Mappings) Apply(state, mp);
    }

   private:
    DeviceTensor* Running(const std::string& key) {
        for (auto& kv : running_)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    void Update(const std::string& key, const DeviceTensor& x) {
        const int64_t cols = x.last();
        DeviceTensor* r = Running(key);
        const bool first = r == nullptr;
        if (first) {
            running_.emplace_back(key, DeviceTensor({cols}, DType::Float32));
            r = &running_.back().second;
        } else if (r->numel() != cols) {
            throw InvalidOperationException("SmoothQuant: activation feature dim changed for '" + key + "': expected " +
                                            std::to_string(r->numel()) + ", got " + std::to_string(cols) + ".");
        }
        SmoothQuant::UpdateActivationMax(*ctx_, x, *r, !first);
    }
    void Apply(CompressionState& state, const SmoothQuantMapping& mp) {
        const DeviceTensor* x = state.HasLayerActivations ? state.Activation(mp.ActivationKey) : nullptr;
        if (!x) {
            if (!Running(mp.ActivationKey))
                throw InvalidOperationException("SmoothQuant: no activation collected for '" + mp.ActivationKey +
                                                "'. Populate CompressionState.LayerActivations.");
        } else if (!Running(mp.ActivationKey)) {
            Update(mp.ActivationKey, *x);
        }
        const DeviceTensor& actMax = *Running(mp.ActivationKey);
        DeviceTensor& smooth = state.Weight(mp.SmoothWeight);
        if (smooth.dim() != 1)
            throw InvalidOperationException("SmoothQuant: smooth weight '" + mp.SmoothWeight + "' must be 1-D (got rank " +
                                            std::to_string(smooth.dim()) + ").");
        DeviceTensor& balance = state.Weight(mp.BalanceWeight);
        if (balance.dim() != 2)
            throw InvalidOperationException("SmoothQuant: balance weight '" + mp.BalanceWeight +
                                            "' must be 2-D (got rank " + std::to_string(balance.dim()) + ").");
        const int64_t hidden = smooth.shape()[0];
        if (actMax.numel() != hidden)
            throw InvalidOperationException("SmoothQuant: activation hidden dim " + std::to_string(actMax.numel()) +
                                            " does not match smooth weight " + std::to_string(hidden) + ".");
        if (balance.shape()[1] != hidden)
            throw InvalidOperationException("SmoothQuant: balance weight last dim " + std::to_string(balance.shape()[1]) +
                                            " does not match hidden " + std::to_string(hidden) + ".");
        SmoothQuant::ApplyMapping(*ctx_, actMax, smooth, balance, cfg_.SmoothingStrength);
    }

    Context* ctx_;
    SmoothQuantConfig cfg_;
    std::vector<std::pair<std::string, DeviceTensor>> running_;
};

// SparseGPT as a recipe type (the plan, phase-4c-sparsegpt.md:1559-1567,1652-1655): calibration
// as GPTQModifier; OnEnd prunes each observed weight against its site's U and writes it back in
// its own dtype (a weight with no calibration rows stays as it is).
struct SparseGPTConfig {
    float Sparsity = 0.5f;
    int MaskN = 0, MaskM = 0;  // 0:0 unstructured; 2:4 for the N:M structure
    int BlockSize = 128;
    float DampeningFrac = 0.01f;
    std::vector<std::string> Targets, Ignore;
};

class SparseGPTModifier : public ModifierBase {
   public:
    SparseGPTModifier(Context& ctx, SparseGPTConfig config)
        : ModifierBase("SparseGPT", config.Targets, config.Ignore), ctx_(&ctx), cfg_(std::move(config)) {}

    void Observe(const std::string& layerName, const DeviceTensor& x) {
        for (auto& a : acc_)
            if (a.first == layerName + ".weight" || a.first == layerName) a.second->Update(x);
    }

   protected:
    void OnStartCore(CompressionState& state) override {
        if (!state.HasNamedModules)
            throw InvalidOperationException("SparseGPTModifier requires CompressionState.NamedModules to be populated.");
        acc_.clear();
        for (const auto& name : TargetedNames(state)) {
            const std::string suffix = ".weight";
            const bool has = name.size() >= suffix.size() && name.compare(name.size() - suffix.size(), suffix.size(), suffix) == 0;
            const std::string layer = has ? name.substr(0, name.size() - suffix.size()) : name;
            if (!state.HasModule(layer)) continue;
            acc_.emplace_back(name, std::make_unique<HessianAccumulator>(*ctx_, (int)state.Weight(name).last()));
        }
    }
    void OnEndCore(CompressionState& state) override {
        for (auto& a : acc_) {
            if (a.second->SampleCount() == 0) continue;
            const int64_t d = a.second->InFeatures();
            DeviceTensor u({d, d}, DType::Float32);
            Check(llmc_chol_inverse(ctx_->get(), a.second->Data(), d, d, cfg_.DampeningFrac, 1,
                                    static_cast<float*>(u.data()), d, 1));
            DeviceTensor& w = state.Weight(a.first);
            SparseGPTResult r = SparseGPT::Prune(*ctx_, w, u, cfg_.Sparsity, cfg_.MaskN, cfg_.MaskM, cfg_.BlockSize);
            if (w.dtype() == DType::Float32) {
                w = std::move(r.Pruned);
            } else {  // round to the weight's dtype (nearest even, one host round trip), as the plan's .to(dtype)
                w = DeviceTensor::FromHost(r.Pruned.ToHost(), w.shape(), w.dtype());
            }
        }
    }
    void OnFinalizeCore(CompressionState&) override { acc_.clear(); }

   private:
    Context* ctx_;
    SparseGPTConfig cfg_;
    std::vector<std::pair<std::string, std::unique_ptr<HessianAccumulator>>> acc_;
};

// AWQ as a recipe type (algorithm-mapping.md:214-249): per mapping, the running activation
// |x| max (as SmoothQuantModifier), then at OnEnd the grid search on the balance weight and the
// chosen scale applied (smooth /= s when a smooth weight is named, balance *= s).
struct AWQConfig {
    RtnConfig Quant{4, false, QuantizationStrategy::Group, 128};
    int NGrid = 20;
    std::vector<SmoothQuantMapping> Mappings;
    std::vector<std::string> Targets, Ignore;
};

class AWQModifier : public ModifierBase {
   public:
    AWQModifier(Context& ctx, AWQConfig config)
        : ModifierBase("AWQ", config.Targets, config.Ignore), ctx_(&ctx), cfg_(std::move(config)) {}
    // The grid point (1-based) chosen for each balance weight.
    std::vector<std::pair<std::string, int>> Chosen;

   protected:
    void OnInitialize(CompressionState&) override {
        running_.clear();
        Chosen.clear();
    }
    void OnBatchCore(CompressionState& state) override {
        if (!state.HasLayerActivations) return;
        for (const auto& mp : cfg_.Mappings)
            if (const DeviceTensor* x = state.Activation(mp.ActivationKey)) Update(mp.ActivationKey, *x);
    }
    void OnEndCore(CompressionState& state) override {
        for (const auto& mp : cfg_.Mappings) {
            if (!Running(mp.ActivationKey)) {
                const DeviceTensor* x = state.HasLayerActivations ? state.Activation(mp.ActivationKey) : nullptr;
                if (!x) throw InvalidOperationException("AWQ: no activation collected for '" + mp.ActivationKey + "'.");
                Update(mp.ActivationKey, *x);
            }
            DeviceTensor& balance = state.Weight(mp.BalanceWeight);
            const AwqResult r = AWQ::Search(*ctx_, balance, *Running(mp.ActivationKey), cfg_.NGrid, cfg_.Quant);
            Chosen.emplace_back(mp.BalanceWeight, r.BestK);
            const DeviceTensor s = DeviceTensor::FromHost(r.BestScale, {(int64_t)r.BestScale.size()});
            ScaleApply::Apply(*ctx_, s, mp.SmoothWeight.empty() ? nullptr : &state.Weight(mp.SmoothWeight), balance);
        }
    }

   private:
    DeviceTensor* Running(const std::string& key) {
        for (auto& kv : running_)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    void Update(const std::string& key, const DeviceTensor& x) {
        DeviceTensor* r = Running(key);
        const bool first = r == nullptr;
        if (first) {
            running_.emplace_back(key, DeviceTensor({x.last()}, DType::Float32));
            r = &running_.back().second;
        }
        SmoothQuant::UpdateActivationMax(*ctx_, x, *r, !first);
    }

    Context* ctx_;
    AWQConfig cfg_;
    std::vector<std::pair<std::string, DeviceTensor>> running_;
};

// CompressionSession.cs: every modifier initialised and started, each calibration batch handed to
// every modifier's OnBatch, then OnEnd; any exception ends the run as Failed (kept in Failure)
// and the initialised modifiers are finalised either way.  A C++ host has no tensor batches for
// the session to pass through: `forward(state, index)` runs its own forward for batch `index`
// (feeding GPTQModifier::Observe or state.LayerActivations) before the OnBatch calls.
enum class SessionStatus { NotStarted, Running, Completed, Failed };

class CompressionSession {
   public:
    explicit CompressionSession(std::vector<ModifierBase*> modifiers) : modifiers_(std::move(modifiers)) {
        for (auto* m : modifiers_)
            if (!m) throw ArgumentNullException("modifiers must not be null");
    }
    SessionStatus Status() const { return status_; }
    std::exception_ptr Failure() const { return failure_; }

    SessionStatus Run(CompressionState& state, int batches, const std::function<void(CompressionState&, int)>& forward) {
        if (status_ != SessionStatus::NotStarted)
            throw InvalidOperationException("CompressionSession.Run may only be called once.");
        status_ = SessionStatus::Running;
        std::vector<ModifierBase*> initialized;
        try {
            for (auto* m : modifiers_) {
                m->Initialize(state);
                initialized.push_back(m);
            }
            for (auto* m : modifiers_) m->OnStart(state);
            for (int i = 0; i < batches; i++) {
                if (forward) forward(state, i);
                for (auto* m : modifiers_) m->OnBatch(state);
            }
            for (auto* m : modifiers_) m->OnEnd(state);
            status_ = SessionStatus::Completed;
        } catch (...) {
            status_ = SessionStatus::Failed;
            failure_ = std::current_exception();
        }
        for (auto* m : initialized) {
            try {
                m->Finalize(state);
            } catch (...) {
                if (status_ != SessionStatus::Failed) throw;  // kept: the run's own failure wins
            }
        }
        return status_;
    }

   private:
    std::vector<ModifierBase*> modifiers_;
    SessionStatus status_ = SessionStatus::NotStarted;
    std::exception_ptr failure_;
};

}  // namespace llmcs

#endif  // LLMC_B200_HPP
