// moe_b200.hpp — C++17 host-side mirror of the reference's MoE operator
// surface, header-only, over the C ABI in moe_b200.h.
//
// Mirrors happyme531/open_rknpu2_lm_infer src/npu.rs (QuantMatrix, Handle,
// check) and src/npu/moe.rs (Backend::load_moe / load_moe_with_shared /
// load_moe_full_k, Moe::run / run_profiled / max_rows / weight_bytes):
// the same names, argument meaning and error behaviour. `ensure!` failures
// throw std::invalid_argument with the reference's message; native failures
// throw moe_b200::Error carrying the library code and its strerror text
// ("{name}: {detail} ({rc})", src/npu.rs:187-193).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "moe_b200.h"

namespace moe_b200 {

struct Error : std::runtime_error {
    int code;
    Error(const std::string& what, int rc)
        : std::runtime_error(what + ": " + moe_b200_strerror(rc) + " (" + std::to_string(rc) + ")"),
          code(rc) {}
};

inline void check(int rc, const char* name) {
    if (rc != MOE_B200_OK) throw Error(name, rc);
}

inline void ensure(bool ok, const char* msg) {
    if (!ok) throw std::invalid_argument(msg);
}

// QuantMatrix (src/npu.rs:135-157) + group-32 fp16 scale extension.
struct QuantMatrix {
    uint32_t bits = 4;
    size_t k = 0, n = 0;
    std::vector<int8_t> codes;          // [k][n]
    std::vector<float> scales;          // [n] (per channel)
    std::vector<uint16_t> group_scales; // [k/32][n] fp16 bits (group = 32)
    int group = 0;

    void validate() const {
        ensure(bits == 4 || bits == 8, "linear weights must use 4 or 8 bits");
        ensure(k > 0 && n > 0 && k <= INT32_MAX && n <= INT32_MAX, "invalid linear dimensions");
        ensure(codes.size() == k * n, "linear weight shape mismatch");
        if (group) {
            ensure(group == 32 && bits == 4 && k % 32 == 0 && group_scales.size() == k / 32 * n,
                   "linear weight shape mismatch");
        } else {
            ensure(scales.size() == n, "linear weight shape mismatch");
        }
    }
    int format() const {
        if (group) return MOE_B200_W4_G32_FP16;
        return bits == 4 ? MOE_B200_W4_PER_CHANNEL : MOE_B200_W8_PER_CHANNEL;
    }
};

// Handle<T> (src/npu.rs:163-186): owns one native object.
template <typename T>
class Handle {
   public:
    Handle() = default;
    Handle(T* raw, void (*free)(T*), const char* name) : raw_(raw), free_(free) {
        if (!raw_) throw Error(std::string("cannot allocate ") + name, MOE_B200_ERR_NOMEM);
    }
    Handle(Handle&& o) noexcept : raw_(std::exchange(o.raw_, nullptr)), free_(o.free_) {}
    Handle& operator=(Handle&& o) noexcept {
        reset();
        raw_ = std::exchange(o.raw_, nullptr);
        free_ = o.free_;
        return *this;
    }
    Handle(const Handle&) = delete;
    Handle& operator=(const Handle&) = delete;
    ~Handle() { reset(); }
    T* get() const { return raw_; }

   private:
    void reset() {
        if (raw_ && free_) free_(raw_);
        raw_ = nullptr;
    }
    T* raw_ = nullptr;
    void (*free_)(T*) = nullptr;
};

using Timings = moe_b200_timings;

class Backend;

// npu::Moe (src/npu/moe.rs:10-14, 242-388).
class Moe {
   public:
    size_t max_rows() const { return (size_t)moe_b200_max_rows(work_); }
    uint64_t weight_bytes() const { return moe_b200_weights_device_bytes(weights_.get()); }

    // Moe::run: host buffers, synchronous. output = routed combine (+ shared).
    void run(const float* input, size_t input_len, const int32_t* ids, size_t ids_len,
             const float* routes, size_t routes_len, float* output, size_t output_len,
             size_t rows) const {
        execute(input, input_len, ids, ids_len, routes, routes_len, output, output_len, rows,
                nullptr);
    }
    // Moe::run_profiled: same call, stage timings from CUDA events.
    Timings run_profiled(const float* input, size_t input_len, const int32_t* ids, size_t ids_len,
                         const float* routes, size_t routes_len, float* output, size_t output_len,
                         size_t rows) const {
        Timings t{};
        execute(input, input_len, ids, ids_len, routes, routes_len, output, output_len, rows, &t);
        return t;
    }
    // Router-inclusive forward on host buffers; output = residual + (routed + shared).
    void forward(const moe_b200_router* router, size_t rows, const float* input,
                 const float* residual, float* output, int32_t* ids = nullptr,
                 float* routes = nullptr, Timings* t = nullptr) const {
        check(moe_b200_forward_f32(work_, weights_.get(), router, (int32_t)rows, input, residual,
                                   output, ids, routes, t),
              "MoE forward");
    }
    // Device pointers, asynchronous on `stream` (cudaStream_t).
    void run_device(size_t rows, const float* d_in, const int32_t* d_ids, const float* d_routes,
                    float* d_out, void* stream) const {
        check(moe_b200_run_device(work_, weights_.get(), (int32_t)rows, d_in, d_ids, d_routes,
                                  d_out, stream),
              "grouped routed FFN");
    }

   private:
    friend class Backend;
    Moe(Handle<moe_b200_weights> w, moe_b200_workspace* work, size_t hidden, size_t top)
        : weights_(std::move(w)), work_(work), hidden_(hidden), top_(top) {}

    void execute(const float* input, size_t input_len, const int32_t* ids, size_t ids_len,
                 const float* routes, size_t routes_len, float* output, size_t output_len,
                 size_t rows, Timings* t) const {
        ensure(input_len == rows * hidden_ && output_len == rows * hidden_ &&
                   ids_len == rows * top_ && routes_len == ids_len,
               "grouped MoE input shape mismatch");
        check(moe_b200_run_f32(work_, weights_.get(), (int32_t)rows, input, ids, routes, output, t),
              "grouped routed FFN");
    }

    Handle<moe_b200_weights> weights_;
    moe_b200_workspace* work_;
    size_t hidden_, top_;
};

// npu::Backend reduced to the MoE surface. Workspaces are shared by every
// bank with the same geometry key (src/npu/moe.rs:198-212).
class Backend {
   public:
    explicit Backend(int device = 0, size_t chunk = 128) : device_(device), chunk_(chunk) {}

    Moe load_moe(const std::vector<QuantMatrix>& gate, const std::vector<QuantMatrix>& down,
                 size_t top) {
        return load(gate, down, top, nullptr, MOE_B200_SHARED_DENSE);
    }
    Moe load_moe_with_shared(const std::vector<QuantMatrix>& gate,
                             const std::vector<QuantMatrix>& down, size_t top,
                             const std::pair<QuantMatrix, QuantMatrix>& shared) {
        const bool joint = shared.first.bits == 8 && shared.first.n == gate.at(0).n;
        return load(gate, down, top, &shared, joint ? MOE_B200_SHARED_JOINT : MOE_B200_SHARED_DENSE);
    }
    Moe load_moe_full_k(const std::vector<QuantMatrix>& gate, const std::vector<QuantMatrix>& down,
                        size_t top) {
        return load_moe(gate, down, top);
    }

    // Router over weight [experts][hidden] (src/model/qwen35/moe.rs:215-241).
    Handle<moe_b200_router> router(const std::vector<float>& weight, size_t experts, size_t hidden,
                                   size_t top, const float* bias = nullptr,
                                   int order = MOE_B200_ROUTER_NEON16, float min_weight = 0.0f) {
        ensure(weight.size() == experts * hidden, "MoE router shape mismatch");
        ensure(top > 0 && top <= experts, "invalid router top-k");
        moe_b200_config cfg = config(hidden, 32, experts, false, top, 0);
        return Handle<moe_b200_router>(
            moe_b200_router_create(&cfg, weight.data(), bias, order, min_weight),
            moe_b200_router_free, "MoE router");
    }

    uint64_t weight_bytes() const { return weight_bytes_; }

   private:
    using Key = std::tuple<size_t, size_t, size_t, size_t, bool, size_t>;

    moe_b200_config config(size_t h, size_t f, size_t e, bool shared, size_t top, size_t is) const {
        moe_b200_config cfg;
        moe_b200_config_init(&cfg, (int32_t)h, (int32_t)f, (int32_t)e, shared ? 1 : 0, (int32_t)top,
                             (int32_t)chunk_);
        cfg.weights.shared_intermediate = (int32_t)is;
        cfg.device = device_;
        return cfg;
    }

    static moe_b200_expert expert(const QuantMatrix& g, const QuantMatrix& d) {
        moe_b200_expert x{};
        x.gate_up = g.codes.data();
        x.down = d.codes.data();
        x.gate_up_scales = g.group ? nullptr : g.scales.data();
        x.down_scales = d.group ? nullptr : d.scales.data();
        x.gate_up_group_scales = g.group ? g.group_scales.data() : nullptr;
        x.down_group_scales = d.group ? d.group_scales.data() : nullptr;
        return x;
    }

    Moe load(const std::vector<QuantMatrix>& gate, const std::vector<QuantMatrix>& down,
             size_t top, const std::pair<QuantMatrix, QuantMatrix>* shared, int mode) {
        ensure(!gate.empty() && gate.size() == down.size(), "invalid expert bank");
        for (const auto& m : gate) m.validate();
        for (const auto& m : down) m.validate();
        const int fmt = gate[0].format();
        for (const auto& m : gate) ensure(m.format() == fmt, "grouped MoE requires one weight format");
        for (const auto& m : down) ensure(m.format() == fmt, "grouped MoE requires one weight format");
        const size_t h = gate[0].k, f = gate[0].n / 2, e = gate.size();
        for (const auto& g : gate) ensure(g.k == h && g.n == 2 * f, "incompatible expert matrices");
        for (const auto& d : down) ensure(d.k == f && d.n == h, "incompatible expert matrices");
        size_t is = 0;
        std::vector<moe_b200_expert> experts;
        for (size_t i = 0; i < e; ++i) experts.push_back(expert(gate[i], down[i]));
        moe_b200_format format{fmt, MOE_B200_W8_PER_CHANNEL, mode};
        if (shared) {
            shared->first.validate();
            shared->second.validate();
            ensure(!shared->first.group && !shared->second.group &&
                       shared->first.bits == shared->second.bits && shared->first.k == h &&
                       shared->second.k == shared->first.n / 2 && shared->second.n == h,
                   "incompatible shared expert matrices");
            is = shared->first.n / 2;
            ensure(mode != MOE_B200_SHARED_JOINT || (shared->first.bits == 8 && is == f),
                   "joint MoE requires a shared W8 expert with the routed intermediate width");
            format.shared_format = shared->first.bits == 8 ? MOE_B200_W8_PER_CHANNEL
                                                           : MOE_B200_W4_PER_CHANNEL;
            experts.push_back(expert(shared->first, shared->second));
        }
        moe_b200_config cfg = config(h, f, e, shared != nullptr, top, is);
        Handle<moe_b200_weights> weights(moe_b200_weights_create(&cfg, experts.data(), &format),
                                         moe_b200_weights_free, "packed MoE expert bank");
        const Key key{h, f, e, top, shared != nullptr, is};
        auto it = work_.find(key);
        if (it == work_.end()) {
            Handle<moe_b200_workspace> ws(moe_b200_workspace_create(&cfg), moe_b200_workspace_free,
                                          "grouped MoE workspace");
            it = work_.emplace(key, std::move(ws)).first;
        }
        weight_bytes_ += moe_b200_weights_device_bytes(weights.get());
        return Moe(std::move(weights), it->second.get(), h, top);
    }

    int device_;
    size_t chunk_;
    std::map<Key, Handle<moe_b200_workspace>> work_;
    uint64_t weight_bytes_ = 0;
};

}  // namespace moe_b200
