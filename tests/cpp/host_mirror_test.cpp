// Exercises the C++ host mirror (include/moe_b200.hpp) against the CPU
// restatement (oracle/moe_oracle.h) on a small deterministic W4 bank, the way
// the reference's own Rust code drives npu::Moe (src/npu/moe.rs:324-333).
// Exit code 0 = all checks passed. Needs an sm_100 GPU.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../include/moe_b200.hpp"
#include "../../oracle/moe_oracle.h"

using moe_b200::QuantMatrix;

static uint32_t lcg(uint32_t& s) { return s = s * 1664525u + 1013904223u; }

static QuantMatrix make(uint32_t& s, size_t k, size_t n, bool group) {
    QuantMatrix m;
    m.bits = 4;
    m.k = k;
    m.n = n;
    m.codes.resize(k * n);
    for (auto& c : m.codes) c = (int8_t)((lcg(s) >> 16) % 16) - 8;
    if (group) {
        m.group = 32;
        m.group_scales.resize(k / 32 * n);
        for (auto& g : m.group_scales)
            g = oracle_float_to_half(0.001f + 0.002f * ((lcg(s) >> 8) % 1000) / 1000.0f);
    } else {
        m.scales.resize(n);
        for (auto& f : m.scales) f = 0.001f + 0.002f * ((lcg(s) >> 8) % 1000) / 1000.0f;
    }
    return m;
}

static oracle_qmat view(const QuantMatrix& m) {
    oracle_qmat q{};
    q.bits = (int)m.bits;
    q.k = (int)m.k;
    q.n = (int)m.n;
    q.group = m.group;
    q.codes = m.codes.data();
    q.scales = m.group ? nullptr : m.scales.data();
    q.gscales = m.group ? m.group_scales.data() : nullptr;
    return q;
}

int main() {
    const size_t H = 256, I = 128, E = 8, K = 2, T = 24;
    int fails = 0;
    for (int group = 0; group < 2; ++group) {
        uint32_t s = 12345 + group;
        std::vector<QuantMatrix> gate, down;
        for (size_t e = 0; e < E; ++e) {
            gate.push_back(make(s, H, 2 * I, group));
            down.push_back(make(s, I, H, group));
        }
        std::vector<float> x(T * H), out(T * H), ref(T * H);
        for (auto& v : x) v = ((lcg(s) >> 8) % 2001) / 1000.0f - 1.0f;
        std::vector<int32_t> ids(T * K);
        std::vector<float> routes(T * K);
        for (size_t t = 0; t < T; ++t) {
            ids[t * K] = (int32_t)(t % E);
            ids[t * K + 1] = (int32_t)((t * 3 + 1) % E);
            routes[t * K] = 0.7f;
            routes[t * K + 1] = t % 5 == 0 ? 0.0f : 0.3f;
        }
        moe_b200::Backend backend(0, T);
        moe_b200::Moe moe = backend.load_moe(gate, down, K);
        auto t = moe.run_profiled(x.data(), x.size(), ids.data(), ids.size(), routes.data(),
                                  routes.size(), out.data(), out.size(), T);
        std::vector<oracle_qmat> og, od;
        for (size_t e = 0; e < E; ++e) {
            og.push_back(view(gate[e]));
            od.push_back(view(down[e]));
        }
        oracle_layer L{};
        L.hidden = (int)H;
        L.inter = (int)I;
        L.experts = (int)E;
        L.top = (int)K;
        L.gate_up = og.data();
        L.down = od.data();
        if (oracle_moe_run(&L, (int)T, x.data(), ids.data(), routes.data(), ref.data(), nullptr)) {
            std::printf("oracle failed\n");
            return 2;
        }
        size_t bad = 0;
        for (size_t i = 0; i < out.size(); ++i)
            if (std::fabs(out[i] - ref[i]) > 1e-3f + 1e-2f * std::fabs(ref[i])) ++bad;
        std::printf("group=%d mismatches=%zu total_us=%.1f max_rows=%zu\n", group, bad, t.total_us,
                    moe.max_rows());
        fails += bad != 0;
        // reference error behaviour: shape mismatch -> ensure!, bad id -> native error
        try {
            moe.run(x.data(), x.size() - 1, ids.data(), ids.size(), routes.data(), routes.size(),
                    out.data(), out.size(), T);
            ++fails;
        } catch (const std::invalid_argument&) {
        }
        ids[3] = (int32_t)E;
        try {
            moe.run(x.data(), x.size(), ids.data(), ids.size(), routes.data(), routes.size(),
                    out.data(), out.size(), T);
            ++fails;
        } catch (const moe_b200::Error& e) {
            if (e.code != MOE_B200_ERR_BAD_EXPERT) ++fails;
        }
        try {
            std::vector<QuantMatrix> g2(gate.begin(), gate.end() - 1);
            backend.load_moe(g2, down, K);
            ++fails;
        } catch (const std::invalid_argument&) {
        }
    }
    std::printf(fails ? "FAILED\n" : "OK\n");
    return fails ? 1 : 0;
}
