// C ABI of the B200 MoE operator (include/moe_b200.h): weight packing,
// workspaces, router objects and the stage orchestration of one MoE call.
//
// Replaces the grouped-MoE operator behind src/npu/moe.rs (Backend::load_moe*,
// Moe::run) of happyme531/open_rknpu2_lm_infer. The call sequence of one run:
//   route_count -> route_scatter -> quant_gather          (dispatch)
//   gemm<gate/up, SwiGLU> -> requant -> gemm<down>         (routed experts)
//   [shared expert: quantise -> gemm -> requant -> gemm]
//   combine (+ shared + residual)
#include <cudaTypedefs.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cmath>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <type_traits>
#include <functional>
#include <vector>

#include "../../include/moe_b200.h"
#include "kernels.cuh"

using namespace moe;

namespace {

// ---- allocation with optional host-side failure injection -----------------
// MOE_B200_FAIL_ALLOC_AFTER=N makes the N-th device allocation (counted from
// process start, 1-based) fail with MOE_B200_ERR_NOMEM, like the reference's
// workspace fault shim (tests/board/workspace_fault_ioctl.c:21-62).
std::mutex g_alloc_mu;
long g_alloc_count = 0;

cudaError_t dev_alloc(void** p, size_t bytes) {
    {
        std::lock_guard<std::mutex> lk(g_alloc_mu);
        ++g_alloc_count;
        const char* env = getenv("MOE_B200_FAIL_ALLOC_AFTER");
        if (env && atol(env) > 0 && g_alloc_count == atol(env)) {
            *p = nullptr;
            return cudaErrorMemoryAllocation;
        }
    }
    if (bytes == 0) bytes = 16;
    return cudaMalloc(p, bytes);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

int cuda_rc(cudaError_t e) {
    if (e == cudaSuccess) return MOE_B200_OK;
    if (e == cudaErrorMemoryAllocation) return MOE_B200_ERR_NOMEM;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver || e == cudaErrorNoKernelImageForDevice)
        return MOE_B200_ERR_NO_DEVICE;
    return MOE_B200_ERR_CUDA;
}

int check_device(int dev, int* num_sms) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || dev < 0 || dev >= count)
        return MOE_B200_ERR_NO_DEVICE;
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10) return MOE_B200_ERR_NO_DEVICE;  // built for sm_100a only
    if (num_sms) cudaDeviceGetAttribute(num_sms, cudaDevAttrMultiProcessorCount, dev);
    return MOE_B200_OK;
}

int pad_to(int v, int m) { return (v + m - 1) / m * m; }

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Tensor map over an int8 row-major [rows][cols] buffer viewed in 3-D as
// (byte within a 128-byte k-block, row, k-block), box = 128 B x nt rows x kKPS
// k-blocks, 128-byte swizzle: one copy lands the MMA operand tiles of all
// k-blocks of a stage, each nt x 128 B and 1024-byte aligned.
int make_act_map(CUtensorMap* map, const void* base, int rows, int cols, int nt) {
    auto enc = get_encode();
    if (!enc || cols % kKAlign) return MOE_B200_ERR_CUDA;
    cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(cols / 128)};
    cuuint64_t strides[2] = {(cuuint64_t)cols, 128};
    cuuint32_t box[3] = {128, (cuuint32_t)nt, (cuuint32_t)kKPS};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MOE_B200_OK : MOE_B200_ERR_CUDA;
}

// The same over an fp16 copy: 64 elements per 128-byte swizzle row, box =
// 64 x nt rows x 4 = the 256 k of one group-32 stage.
int make_act_map_h(CUtensorMap* map, const void* base, int rows, int cols, int nt) {
    auto enc = get_encode();
    if (!enc || cols % kKAlign) return MOE_B200_ERR_CUDA;
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)nt, (cuuint32_t)(2 * kKPS)};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MOE_B200_OK : MOE_B200_ERR_CUDA;
}

constexpr int kNTs[3] = {16, 32, 64};
int nt_index(int nt) { return nt == 16 ? 0 : nt == 32 ? 1 : 2; }
// Token tile (MMA N) from the expected rows per expert. An MMA costs the same
// for N <= 64, so tiles grow to 64 once an expert averages more than 16 rows.
int choose_nt(long rows, int experts) {
    const long avg = experts > 0 ? (rows + experts - 1) / experts : rows;
    if (avg <= 8) return 16;
    if (avg <= 16) return 32;
    return 64;
}
// The exact int8 group-32 kernel keeps four K=32 buffers per k-block in TMEM,
// which caps its tile at 32 tokens.
int exact_nt(int nt, int fmt) { return fmt == kFmtW4G32 && nt > 32 ? 32 : nt; }
// Group-32 down projections keep exact group sums unless the bank opted into
// the fp16 tensor cores (MOE_B200_W4_G32_FP16_ROUNDED_DOWN); gate/up
// projections always keep the exact per-group sums.
int down_fmt(int fmt, bool exact) { return fmt == kFmtW4G32 && !exact ? kFmtW4G32H : fmt; }

// ---- packed matrices ------------------------------------------------------

struct PackedMat {
    uint8_t* w = nullptr;
    void* s = nullptr;
    size_t w_expert_stride = 0, w_tile_stride = 0, w_stage_stride = 0;
    size_t s_expert_stride = 0, s_tile_stride = 0;
    int fmt = 0, kblocks = 0, row_tiles = 0, experts = 0;
    int k = 0, n = 0;        // logical K and output channels (n = I for SwiGLU)
    bool swiglu = false;
};

// Byte offset of element (row, kbyte) in a 128-row x 128-byte operand tile
// stored in the 128-byte swizzle layout (8-row atoms of 1024 bytes, 16-byte
// chunk index XOR row%8).
inline size_t sw128(int row, int kbyte) {
    return (size_t)(row / 8) * 1024 + (row % 8) * 128 + (((kbyte / 16) ^ (row % 8)) * 16) +
           (kbyte % 16);
}

// Weight channel held by tile row lr of row tile rt, or -1 for padding.
inline int tile_channel(const PackedMat& m, int rt, int lr) {
    if (m.swiglu) {
        const int c = rt * 64 + (lr & 63);
        if (c >= m.n) return -1;
        return lr < 64 ? c : m.n + c;  // gate columns first, then up (concatenate order)
    }
    const int c = rt * 128 + lr;
    return c < m.n ? c : -1;
}

// Group-32 stage: 256 k of 128 rows = 16 KB of nibbles (row r: 128 bytes, its
// 16-byte chunk c at position c ^ (r & 7), conflict-free for one row per
// thread) followed by the rows' 8 group scales (fp16, 16 bytes per row).
// Chunk c is group c of the stage; its word w holds k = 32c + 8w + j with j
// even in nibble j/2 and j odd in nibble 4 + j/2 as the offset-binary code
// w + 8, so one mask of 0x000F000F after a shift by 4i yields the fp16 pair
// (k = 2i, 2i + 1) and byte permutes yield int8 in k order.
constexpr size_t kG32StageW = 128 * 128;
constexpr size_t kG32Stage = kG32StageW + 128 * 16;

// Packs one reference-layout matrix (codes [K][N], N = 2n for SwiGLU) into
// tile-major device order, per 128-row tile and load stage (kKPS k-blocks of
// 128 k). Per-channel formats: the stage's weight blocks (W8: the tensor
// core's 128-byte-swizzle K-major layout; W4: 64 bytes per row, 16-byte chunk
// c (k 32c..32c+31) at chunk c ^ ((r >> 1) & 3), byte b of word w holding k =
// 32c+8w+b in its low nibble and k+4 in its high nibble), f32 scales [128] per
// tile in host_s. Group-32: the stage layout above. host_w / host_s point at
// this expert's slot.
void pack_expert(const PackedMat& m, const int8_t* codes, const float* scales,
                 const uint16_t* gscales, uint8_t* host_w, uint8_t* host_s) {
    const int K = m.k;
    const int N = m.swiglu ? 2 * m.n : m.n;
    const bool w4 = m.fmt != kFmtW8PC;
    const size_t tile_bytes = w4 ? 8192 : 16384;
    for (int rt = 0; rt < m.row_tiles; ++rt) {
        for (int lr = 0; lr < 128; ++lr) {
            const int ch = tile_channel(m, rt, lr);
            for (int kb = 0; kb < m.kblocks; ++kb) {
                uint8_t* stage = host_w + (size_t)rt * m.w_tile_stride + (kb / kKPS) * m.w_stage_stride;
                uint8_t* tile = stage + (size_t)(kb % kKPS) * tile_bytes;
                for (int kbyte = 0; kbyte < 128; ++kbyte) {
                    const int k = kb * 128 + kbyte;
                    const int8_t code = (ch >= 0 && k < K) ? codes[(size_t)k * N + ch] : 0;
                    if (m.fmt == kFmtW4G32) {
                        const int ks = (kb % kKPS) * 128 + kbyte;  // k within the stage
                        const int c = ks / 32, w = (ks % 32) / 8, j = ks % 8;
                        const int p = (j & 1) ? 4 + j / 2 : j / 2;
                        const size_t pb = (size_t)lr * 128 + ((c ^ (lr & 7)) * 16) + w * 4 + p / 2;
                        const uint8_t nib = (uint8_t)((code + 8) & 0xF);
                        stage[pb] = (p & 1) ? (uint8_t)((stage[pb] & 0x0F) | (nib << 4))
                                            : (uint8_t)((stage[pb] & 0xF0) | nib);
                    } else if (!w4) {
                        tile[sw128(lr, kbyte)] = (uint8_t)code;
                    } else {
                        const int c = kbyte / 32, w = (kbyte % 32) / 8, e = kbyte % 8;
                        const size_t pb = (size_t)lr * 64 + ((c ^ ((lr >> 1) & 3)) * 16) + w * 4 + (e & 3);
                        const uint8_t nib = (uint8_t)code & 0xF;
                        if (e < 4)
                            tile[pb] = (uint8_t)((tile[pb] & 0xF0) | nib);
                        else
                            tile[pb] = (uint8_t)((tile[pb] & 0x0F) | (nib << 4));
                    }
                }
                if (m.fmt == kFmtW4G32) {
                    uint16_t* st = reinterpret_cast<uint16_t*>(stage + kG32StageW + (size_t)lr * 16);
                    for (int j = 0; j < 4; ++j) {
                        const int g = kb * 4 + j;
                        st[(kb % kKPS) * 4 + j] =
                            (ch >= 0 && g * 32 < K) ? gscales[(size_t)g * N + ch] : (uint16_t)0;
                    }
                }
            }
            if (m.fmt != kFmtW4G32) {
                float* st = reinterpret_cast<float*>(host_s + (size_t)rt * m.s_tile_stride);
                st[lr] = ch >= 0 ? scales[ch] : 0.0f;
            }
        }
    }
}

int setup_mat(PackedMat& m, int fmt, int experts, int K, int n, bool swiglu) {
    m.fmt = fmt;
    m.experts = experts;
    m.k = K;
    m.n = n;
    m.swiglu = swiglu;
    m.kblocks = pad_to(K, kKAlign) / 128;
    m.row_tiles = swiglu ? (n + 63) / 64 : (n + 127) / 128;
    const size_t tile_bytes = fmt == kFmtW8PC ? 16384 : 8192;
    const size_t stages = (size_t)(m.kblocks / kKPS);
    static_assert(kKPS == 2, "group-32 stages hold 256 k (8 groups)");
    m.w_stage_stride = fmt == kFmtW4G32 ? kG32Stage : kKPS * tile_bytes;
    m.w_tile_stride = stages * m.w_stage_stride;
    m.w_expert_stride = (size_t)m.row_tiles * m.w_tile_stride;
    m.s_tile_stride = 512;  // per-channel f32 scales of one tile (group scales live in w)
    m.s_expert_stride = (size_t)m.row_tiles * m.s_tile_stride;
    return MOE_B200_OK;
}

}  // namespace

// ---- opaque objects ---------------------------------------------------------

// Creation serials: a bank or router freed and another created at the same
// address never matches a graph captured over the first.
static std::atomic<uint64_t> g_serial{0};

struct moe_b200_weights {
    uint64_t serial = ++g_serial;
    int device = 0;
    int H = 0, I = 0, E = 0, shared = 0, Is = 0, top = 0;
    int shared_mode = MOE_B200_SHARED_DENSE;
    bool exact_down = false;  // group-32: down GEMM on exact int32 group sums too
    PackedMat gu, dn, sgu, sdn;
    uint64_t bytes = 0;
};

struct moe_b200_router {
    uint64_t serial = ++g_serial;
    int device = 0, H = 0, E = 0, order = 0;
    float min_weight = 0.0f;
    float* w = nullptr;     // [E (+1 gate row)][H]
    float* bias = nullptr;
    int rule = 0, groups = 1, top_groups = 1;
    float scale = 1.0f;
    float* sel_bias = nullptr;
    bool gate = false;      // row E of w is the shared-expert gate
    int rows() const { return E + (gate ? 1 : 0); }
};

struct moe_b200_workspace {
    int device = 0, H = 0, I = 0, E = 0, k = 0, max_rows = 0, Is = 0, num_sms = 0;
    int Kh = 0, Ki = 0, Kis = 0;
    long n_max = 0;
    std::vector<void*> allocs;
    uint64_t bytes = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t copy_stream = nullptr;  // host-API residual upload, overlapped with the layer
    // small-batch layers of banks with a shared expert: the shared FFN runs on
    // a side stream beside the routed GEMVs (fork / join events)
    cudaStream_t side_stream = nullptr;
    cudaEvent_t side_fork = nullptr, side_join = nullptr;
    // host-buffer calls: a pinned word for the status read with the outputs,
    // and the last call's copies + layer captured as a CUDA graph (replayed
    // while the call's buffers, bank, router and row count stay the same)
    uint32_t* h_err = nullptr;
    struct HostGraph {
        uint64_t key[12] = {};
        int rows = 0;
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        int64_t launches = 0;
        bool failed = false;  // these buffers did not capture: run them eagerly
    } hg;
    cudaEvent_t res_ready = nullptr;
    cudaEvent_t x_ready = nullptr;  // host-API input upload done (orders the residual's after it)
    cudaStream_t last_stream = nullptr;
    // staging for the host-pointer API
    float *x = nullptr, *out = nullptr, *res = nullptr, *routes = nullptr;
    int32_t* ids = nullptr;
    // dispatch
    int8_t* q_x = nullptr;
    float* s_x = nullptr;
    int32_t *hist = nullptr, *offsets = nullptr, *perm = nullptr, *pos = nullptr;
    int32_t *shared_offsets = nullptr, *counters = nullptr;
    int32_t* gv_counters = nullptr;  // small-batch path: last-arrival counters
    // fused small-batch layer: the grid barrier's counters (dec_bar), and
    // [n_max] middle-row max bits + [n_max] gate/up items done per assignment
    uint32_t* dec_state = nullptr;
    unsigned long long* dec_bar = nullptr;  // [8 x 16]: eight counters 128 bytes apart
    bool coop = false;  // the device runs cooperative launches
    int8_t* a_perm = nullptr;
    __half *q_m_h = nullptr, *sq_m_h = nullptr;  // fp16 copies of the middle codes (group-32 down)
    float* s_perm = nullptr;
    // routed experts
    float* gate_up = nullptr;  // dequantised gate | up rows [n][2I]
    int8_t* q_m = nullptr;
    float *s_m = nullptr, *y = nullptr;

    // shared expert
    int8_t *q_xd = nullptr, *sq_m = nullptr;
    float *s_xd = nullptr, *s_middle = nullptr, *ss_m = nullptr, *s_y = nullptr;
    // small-batch shared FFN of per-channel int8 banks (split-K GEMVs):
    // int32 accumulators, last-arrival counters, middle row maxima
    int32_t* w8_acc = nullptr;
    int* w8_cnt = nullptr;
    uint32_t* w8_max = nullptr;
    // small-batch routed experts of per-channel int8 banks (split-K GEMVs)
    int32_t* w8r_acc = nullptr;
    int* w8r_cnt = nullptr;
    uint32_t* w8r_max = nullptr;
    size_t w8r_acc_n = 0, w8r_cnt_n = 0;
    float* logits = nullptr;
    uint32_t* err = nullptr;
    CUtensorMap map_a[3], map_qm[3], map_qx[3], map_qxd[3], map_sqm[3];
    CUtensorMap map_qm_h[3], map_sqm_h[3];
    cudaEvent_t ev[12] = {};
    // stage-profiling ring of device calls
    static constexpr int kProfSlots = 64, kProfEvents = 9;
    bool profiling = false;
    int prof_calls = 0;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_flags;  // bit0 router ran, bit1 shared ran
    int64_t launches = 0;
    // last call, for accumulator dumps
    int last_rows = 0;
    int last_logit_cols = 0;  // logits row stride of the last routing call
    int last_nt_gu = 16, last_nt_dn = 16;
    const moe_b200_weights* last_w = nullptr;
};

namespace {

template <typename T>
int ws_alloc(moe_b200_workspace* ws, T** p, size_t count) {
    void* v = nullptr;
    const size_t bytes = sizeof(T) * (count > 0 ? count : 1);
    cudaError_t e = dev_alloc(&v, bytes);
    if (e != cudaSuccess) return MOE_B200_ERR_NOMEM;
    ws->allocs.push_back(v);
    ws->bytes += bytes;
    *p = static_cast<T*>(v);
    return MOE_B200_OK;
}

int map_err_bits(uint32_t bits) {
    if (bits & kErrWaitTimeout) return MOE_B200_ERR_DEVICE_TIMEOUT;
    if (bits & kErrBadExpert) return MOE_B200_ERR_BAD_EXPERT;
    // a non-finite logit or activation also makes NaN routing weights: report
    // the cause (caller-supplied bad routes set only the route bit)
    if (bits & kErrNonFinite) return MOE_B200_ERR_NONFINITE;
    if (bits & kErrBadRoute) return MOE_B200_ERR_BAD_ROUTE;
    if (bits & kErrCapacity) return MOE_B200_ERR_CAPACITY;
    return MOE_B200_OK;
}

GemmArgs gemm_args(moe_b200_workspace* ws, const PackedMat& m, const float* act_scale,
                   const int32_t* offsets, int experts, long max_rows, float* out, int ldo) {
    GemmArgs a{};
    a.act_scale = act_scale;
    a.offsets = offsets;
    a.num_experts = experts;
    a.max_rows = (int)max_rows;
    a.w = m.w;
    a.w_expert_stride = m.w_expert_stride;
    a.w_tile_stride = m.w_tile_stride;
    a.w_stage_stride = m.w_stage_stride;
    a.wscale = m.s;
    a.ws_expert_stride = m.s_expert_stride;
    a.ws_tile_stride = m.s_tile_stride;
    a.kblocks = m.kblocks;
    a.row_tiles = m.row_tiles;
    a.out = out;
    a.ldo = ldo;
    a.n_valid = m.n;
    a.swiglu_layout = m.swiglu ? 1 : 0;
    a.err = ws->err;
    return a;
}

// Routed gate/up GEMM (gate | up rows) and the middle requantisation (SwiGLU,
// row max, int8 codes). `mark` records the gate/up and middle stage events of
// the profiling ring (index 4 and 5). A SwiGLU + requantisation fused into the
// group-32 GEMM's epilogue was measured slower: its tile tail (an exchange of
// the up values, SwiGLU, a per-token-tile arrival counter) stalls the three
// accumulator slots of the pipeline (c2, 512 tokens: 441 us against 176 + 15).
int run_gate_up(moe_b200_workspace* ws, const moe_b200_weights* w, long n, int nt_g, bool hd,
                cudaStream_t s, const std::function<void(int)>& mark) {
    const int E = ws->E, I = ws->I;
    GemmArgs g = gemm_args(ws, w->gu, ws->s_perm, ws->offsets, E, n, ws->gate_up, 2 * I);
    if (launch_gemm(ws->map_a[nt_index(nt_g)], g, w->gu.fmt, kEpiGateUp, nt_g, ws->num_sms, s))
        return MOE_B200_ERR_UNSUPPORTED;
    mark(4);
    launch_requant(ws->gate_up, ws->offsets + E, (int)n, I, ws->Ki, kQuantMoe, ws->q_m,
                   hd ? ws->q_m_h : nullptr, ws->s_m, s);
    mark(5);
    return MOE_B200_OK;
}

// Shared expert FFN over all rows (joint: reuses q_x; dense: own quantisation).
// Tokens per call of the small-batch paths (the group-32 GEMVs and the
// split-K GEMVs of a shared per-channel int8 bank).
constexpr int kGemvMaxRows = 4;
// Router-inclusive calls of at most this many tokens run as the fused decode
// launch. Graph replays (µs, fused / router + two GEMV kernels): config 2 at
// 1-4 tokens 23.5 / 30.8, 40.9 / 39.0, 51.5 / 41.0, 69.6 / 53.1; config 5's
// routed bank 24.6 / 26.7, 36.7 / 30.2, 47.1 / 36.9, 62.8 / 38.9. From two
// tokens on, the fused kernel's gate/up items outnumber its CTAs and each
// CTA streams its items one after another.
constexpr int kFusedMaxRows = 1;

// Whether the shared FFN of `rows` tokens runs as the split-K GEMVs
// (gemv_w8.cu): a per-channel int8 bank at one to four tokens.
bool shared_gemv(const moe_b200_weights* w, int rows) {
    return rows >= 1 && rows <= kGemvMaxRows && w->sgu.fmt == kFmtW8PC && w->sdn.fmt == kFmtW8PC &&
           w->Is % 4 == 0 && w->H % 4 == 0;
}

int run_shared(moe_b200_workspace* ws, const moe_b200_weights* w, int rows, const float* d_x,
               cudaStream_t s) {
    const int rule = w->shared_mode == MOE_B200_SHARED_JOINT ? kQuantMoe : kQuantDense;
    if (shared_gemv(w, rows)) {
        const bool joint = w->shared_mode == MOE_B200_SHARED_JOINT;
        if (!joint)
            launch_quant_gather(d_x, rows, ws->H, ws->Kh, kQuantDense, 1, nullptr, ws->q_xd, ws->s_xd,
                                nullptr, nullptr, nullptr, nullptr, ws->err, s);
        W8GemvArgs g{};
        g.w = w->sgu.w;
        g.w_tile_stride = w->sgu.w_tile_stride;
        g.w_stage_stride = w->sgu.w_stage_stride;
        g.wscale = w->sgu.s;
        g.ws_tile_stride = w->sgu.s_tile_stride;
        g.q = joint ? ws->q_x : ws->q_xd;
        g.ld = ws->Kh;
        g.sx = joint ? ws->s_x : ws->s_xd;
        g.T = rows;
        g.n = w->Is;
        g.acc = ws->w8_acc;
        g.counters = ws->w8_cnt;
        g.row_max = ws->w8_max;
        g.out = ws->s_middle;
        g.q_out = ws->sq_m;
        g.q_scale = ws->ss_m;
        g.ld_q = ws->Kis;
        g.rule = rule;
        g.err = ws->err;
        if (launch_shared_w8(g, true, w->sgu.row_tiles, w->sgu.kblocks / kKPS, s))
            return MOE_B200_ERR_UNSUPPORTED;
        W8GemvArgs d = g;
        d.w = w->sdn.w;
        d.w_tile_stride = w->sdn.w_tile_stride;
        d.w_stage_stride = w->sdn.w_stage_stride;
        d.wscale = w->sdn.s;
        d.ws_tile_stride = w->sdn.s_tile_stride;
        d.q = ws->sq_m;
        d.ld = ws->Kis;
        d.sx = ws->ss_m;
        d.n = ws->H;
        d.counters = ws->w8_cnt + 512;
        d.out = ws->s_y;
        if (launch_shared_w8(d, false, w->sdn.row_tiles, w->sdn.kblocks / kKPS, s))
            return MOE_B200_ERR_UNSUPPORTED;
        return MOE_B200_OK;
    }
    const int nt = choose_nt(rows, 1);
    const int nt_g = exact_nt(nt, w->sgu.fmt);
    const bool hd = down_fmt(w->sdn.fmt, false) == kFmtW4G32H;
    const CUtensorMap* amap = &ws->map_qx[nt_index(nt_g)];
    const float* ascale = ws->s_x;
    if (w->shared_mode != MOE_B200_SHARED_JOINT) {
        launch_quant_gather(d_x, rows, ws->H, ws->Kh, kQuantDense, 1, nullptr, ws->q_xd, ws->s_xd,
                            nullptr, nullptr, nullptr, nullptr, ws->err, s);
        amap = &ws->map_qxd[nt_index(nt_g)];
        ascale = ws->s_xd;
    }
    GemmArgs g = gemm_args(ws, w->sgu, ascale, ws->shared_offsets, 1, rows, ws->s_middle, 2 * w->Is);
    if (launch_gemm(*amap, g, w->sgu.fmt, kEpiGateUp, nt_g, ws->num_sms, s))
        return MOE_B200_ERR_UNSUPPORTED;
    launch_requant(ws->s_middle, ws->shared_offsets + 1, rows, w->Is, ws->Kis, rule, ws->sq_m,
                   hd ? ws->sq_m_h : nullptr, ws->ss_m, s);
    GemmArgs d = gemm_args(ws, w->sdn, ws->ss_m, ws->shared_offsets, 1, rows, ws->s_y, ws->H);
    if (launch_gemm(hd ? ws->map_sqm_h[nt_index(nt)] : ws->map_sqm[nt_index(nt)], d,
                    down_fmt(w->sdn.fmt, false), kEpiStore, nt, ws->num_sms, s))
        return MOE_B200_ERR_UNSUPPORTED;
    return MOE_B200_OK;
}

// Activation / output rows are moved as 16-byte vectors.
bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int compatible(const moe_b200_workspace* ws, const moe_b200_weights* w) {
    if (!ws || !w) return MOE_B200_ERR_INVALID;
    if (ws->H != w->H || ws->I != w->I || ws->E != w->E || ws->k != w->top ||
        ws->device != w->device)
        return MOE_B200_ERR_INVALID;
    if (w->shared && ws->Is < w->Is) return MOE_B200_ERR_INVALID;
    return MOE_B200_OK;
}

// Event set of the next profiled device call (nullptr when profiling is off).
cudaEvent_t* prof_slot(moe_b200_workspace* ws, int flags) {
    if (!ws->profiling) return nullptr;
    const int slot = ws->prof_calls % moe_b200_workspace::kProfSlots;
    ws->prof_flags[slot] = flags;
    ++ws->prof_calls;
    return &ws->prof_ev[(size_t)slot * moe_b200_workspace::kProfEvents];
}

// The whole routed (+ shared) pipeline on device pointers. ev != null records
// stage events for run_profiled-style timings.
// Small batches of group-32 banks run the GEMV path (csrc/gemv.cu): with
// caller-supplied routes, 2 launches, every weight stage in flight (a shared
// expert beside them on the side stream); router-inclusive calls of banks
// without a shared expert run the whole layer as one cooperative launch
// (decode_layer_kernel, see layer_impl).

bool use_gemv(const moe_b200_workspace* ws, const moe_b200_weights* w, int rows) {
    return rows <= kGemvMaxRows && w->gu.fmt == kFmtW4G32 && w->dn.fmt == kFmtW4G32 &&
           (int)(gemv_smem_bytes((int)(w->gu.kblocks / kKPS))) <= (int)kGemvMaxSmem &&
           gemv_smem_bytes((int)(w->dn.kblocks / kKPS)) <= kGemvMaxSmem && ws->k <= 32;
}

GemvArgs gemv_args(const moe_b200_workspace* ws, const moe_b200_weights* w, int rows,
                   const float* d_x, const int32_t* d_ids, const float* d_routes,
                   const float* d_res, float* d_out);

// Small batches of per-channel int8 routed banks: the split-K GEMVs of
// gemv_w8.cu (gate/up with the token's codes, SwiGLU and the middle's codes;
// down with the combine).
bool use_w8_gemv(const moe_b200_workspace* ws, const moe_b200_weights* w, int rows) {
    return rows >= 1 && rows <= kGemvMaxRows && w->gu.fmt == kFmtW8PC && w->dn.fmt == kFmtW8PC &&
           ws->k <= 32 && ws->H % 4 == 0 && ws->I % 4 == 0;
}

// The shared-gate logits of a gated router: column E of the workspace logits.
struct GateRef {
    const float* logits = nullptr;
    int ld = 0;
};

int run_shared(moe_b200_workspace* ws, const moe_b200_weights* w, int rows, const float* d_x,
               cudaStream_t s);

// The shared expert's FFN of a small batch on the workspace's side stream (its
// own activation quantisation, the one-expert grouping, the tensor-core GEMMs),
// forked from stream s; side_join marks its end. It needs no routing, so a
// router-inclusive call starts it before the router.
int start_shared_side(moe_b200_workspace* ws, const moe_b200_weights* w, int rows,
                      const float* d_x, cudaStream_t s) {
    cudaStream_t side = ws->side_stream;
    cudaEventRecord(ws->side_fork, s);
    cudaStreamWaitEvent(side, ws->side_fork, 0);
    if (shared_gemv(w, rows)) {
        ws->launches += 3;  // quantisation, gate/up (+ requantisation), down
    } else {
        launch_set_range(ws->shared_offsets, rows, side);  // the tensor-core GEMMs' grouping
        ws->launches += 5;  // range, quantisation, gate/up, requantisation, down
    }
    if (w->shared_mode == MOE_B200_SHARED_JOINT)  // the routed rows' MoE A8 codes
        launch_quant_gather(d_x, rows, ws->H, ws->Kh, kQuantMoe, 1, nullptr, ws->q_x, ws->s_x,
                            nullptr, nullptr, nullptr, nullptr, ws->err, side);
    const int rc = run_shared(ws, w, rows, d_x, side);
    cudaEventRecord(ws->side_join, side);
    return rc;
}

int run_small_w8(moe_b200_workspace* ws, const moe_b200_weights* w, int rows, const float* d_x,
                 const int32_t* d_ids, const float* d_routes, const float* d_res, float* d_out,
                 cudaStream_t s, cudaEvent_t* evs, cudaEvent_t res_ready, GateRef gate,
                 bool shared_started) {
    auto mark = [&](int i) {
        if (evs) cudaEventRecord(evs[i], s);
    };
    ws->launches += 2;
    mark(1);
    mark(2);
    mark(3);
    W8RoutedArgs a{};
    a.ids = d_ids;
    a.routes = d_routes;
    a.T = rows;
    a.k = ws->k;
    a.E = ws->E;
    a.H = ws->H;
    a.I = ws->I;
    a.gu_stages = w->gu.kblocks / kKPS;
    a.dn_stages = w->dn.kblocks / kKPS;
    a.x = d_x;
    a.gu_w = w->gu.w;
    a.gu_expert_stride = w->gu.w_expert_stride;
    a.gu_tile_stride = w->gu.w_tile_stride;
    a.gu_stage_stride = w->gu.w_stage_stride;
    a.gu_s = static_cast<const float*>(w->gu.s);
    a.gu_s_expert_stride = w->gu.s_expert_stride;
    a.gu_s_tile_stride = w->gu.s_tile_stride;
    a.dn_w = w->dn.w;
    a.dn_expert_stride = w->dn.w_expert_stride;
    a.dn_tile_stride = w->dn.w_tile_stride;
    a.dn_stage_stride = w->dn.w_stage_stride;
    a.dn_s = static_cast<const float*>(w->dn.s);
    a.dn_s_expert_stride = w->dn.s_expert_stride;
    a.dn_s_tile_stride = w->dn.s_tile_stride;
    a.acc = ws->w8r_acc;
    a.counters = ws->w8r_cnt;
    a.row_max = ws->w8r_max;
    a.middle = ws->gate_up;
    a.q_m = ws->q_m;
    a.s_m = ws->s_m;
    a.ld_qm = ws->Ki;
    a.y = ws->y;
    a.residual = d_res;
    a.out = d_out;
    a.err = ws->err;
    if (w->shared) {
        const int rc = shared_started ? MOE_B200_OK : start_shared_side(ws, w, rows, d_x, s);
        if (rc) {
            cudaStreamWaitEvent(s, ws->side_join, 0);
            return rc;
        }
        a.shared = ws->s_y;
        a.gate = gate.logits;
        a.gate_ld = gate.ld;
    }
    if (launch_routed_w8(a, 0, s)) {
        if (w->shared) cudaStreamWaitEvent(s, ws->side_join, 0);
        return MOE_B200_ERR_UNSUPPORTED;
    }
    mark(4);
    mark(5);
    if (res_ready) cudaStreamWaitEvent(s, res_ready, 0);
    if (w->shared) cudaStreamWaitEvent(s, ws->side_join, 0);
    if (launch_routed_w8(a, 1, s)) return MOE_B200_ERR_UNSUPPORTED;
    mark(6);
    mark(7);
    mark(8);
    ws->last_rows = 0;  // no permuted accumulators to dump for this call
    ws->last_w = w;
    ws->last_stream = s;
    return cuda_rc(cudaPeekAtLastError());
}

// The small-batch layer: the routed experts as two GEMV kernels (gate/up with
// SwiGLU and requantisation, down with the combine). A shared expert's FFN
// runs beside them on the side stream (started here unless the caller already
// did: shared_started) and enters the down kernel's combine after the ranks,
// as in combine_kernel.
int run_small(moe_b200_workspace* ws, const moe_b200_weights* w, int rows, const float* d_x,
              const int32_t* d_ids, const float* d_routes, const float* d_res, float* d_out,
              cudaStream_t s, cudaEvent_t* evs, cudaEvent_t res_ready, GateRef gate = {},
              bool shared_started = false) {
    auto mark = [&](int i) {
        if (evs) cudaEventRecord(evs[i], s);
    };
    ws->launches += 2;
    mark(1);
    mark(2);
    mark(3);
    GemvArgs a = gemv_args(ws, w, rows, d_x, d_ids, d_routes, d_res, d_out);
    if (w->shared) {
        const int rc = shared_started ? MOE_B200_OK : start_shared_side(ws, w, rows, d_x, s);
        if (rc) {
            cudaStreamWaitEvent(s, ws->side_join, 0);
            return rc;
        }
        a.shared = ws->s_y;
        a.gate = gate.logits;
        a.gate_ld = gate.ld;
    }
    if (launch_gemv(a, 0, s)) {
        if (w->shared) cudaStreamWaitEvent(s, ws->side_join, 0);
        return MOE_B200_ERR_UNSUPPORTED;
    }
    mark(4);
    mark(5);
    if (res_ready) cudaStreamWaitEvent(s, res_ready, 0);
    if (w->shared) cudaStreamWaitEvent(s, ws->side_join, 0);
    if (launch_gemv(a, 1, s)) return MOE_B200_ERR_UNSUPPORTED;
    mark(6);
    mark(7);
    mark(8);
    ws->last_rows = 0;  // no permuted accumulators to dump for this call
    ws->last_w = w;
    ws->last_stream = s;
    return cuda_rc(cudaPeekAtLastError());
}

GemvArgs gemv_args(const moe_b200_workspace* ws, const moe_b200_weights* w, int rows,
                   const float* d_x, const int32_t* d_ids, const float* d_routes,
                   const float* d_res, float* d_out) {
    GemvArgs a{};
    a.ids = d_ids;
    a.routes = d_routes;
    a.T = rows;
    a.k = ws->k;
    a.E = ws->E;
    a.H = ws->H;
    a.I = ws->I;
    a.x = d_x;
    a.gu_w = w->gu.w;
    a.gu_expert_stride = w->gu.w_expert_stride;
    a.gu_tile_stride = w->gu.w_tile_stride;
    a.gu_stage_stride = w->gu.w_stage_stride;
    a.gu_stages = w->gu.kblocks / kKPS;
    a.dn_w = w->dn.w;
    a.dn_expert_stride = w->dn.w_expert_stride;
    a.dn_tile_stride = w->dn.w_tile_stride;
    a.dn_stage_stride = w->dn.w_stage_stride;
    a.dn_stages = w->dn.kblocks / kKPS;
    a.middle = ws->gate_up;
    a.q_m = ws->q_m;
    a.s_m = ws->s_m;
    a.ld_qm = ws->Ki;
    a.y = ws->y;
    a.residual = d_res;
    a.out = d_out;
    a.counters = ws->gv_counters;
    a.dn_counter_base = (int)ws->n_max;
    a.err = ws->err;
    return a;
}


int run_pipeline(moe_b200_workspace* ws, const moe_b200_weights* w, int rows, const float* d_x,
                 const int32_t* d_ids, const float* d_routes, const float* d_res, float* d_out,
                 cudaStream_t s, cudaEvent_t* evs, cudaEvent_t res_ready = nullptr,
                 GateRef gate = {}, bool shared_started = false) {
    if (use_gemv(ws, w, rows))
        return run_small(ws, w, rows, d_x, d_ids, d_routes, d_res, d_out, s, evs, res_ready, gate,
                         shared_started);
    if (use_w8_gemv(ws, w, rows))
        return run_small_w8(ws, w, rows, d_x, d_ids, d_routes, d_res, d_out, s, evs, res_ready,
                            gate, shared_started);
    const int E = ws->E, k = ws->k, H = ws->H;
    const long n = (long)rows * k;
    auto mark = [&](int i) {
        if (evs) cudaEventRecord(evs[i], s);
    };
    // route count + scatter (when there are assignments), quantise, gate/up,
    // requantise, down, combine
    ws->launches += (n + kRouteChunk - 1) / kRouteChunk > 0 ? 7 : 5;
    if (w->shared)
        ws->launches += (w->shared_mode == MOE_B200_SHARED_JOINT ? 0 : 1) + (shared_gemv(w, rows) ? 2 : 3);
    mark(1);
    launch_route_count(d_ids, d_routes, (int)n, E, ws->hist, ws->err, s);
    launch_route_scatter(d_ids, d_routes, (int)n, E, ws->hist, ws->offsets, ws->perm, ws->pos,
                         ws->shared_offsets, rows, s);
    mark(2);
    launch_quant_gather(d_x, rows, H, ws->Kh, kQuantMoe, k, ws->pos, ws->q_x, ws->s_x, ws->a_perm,
                        ws->s_perm, nullptr, nullptr, ws->err, s);
    mark(3);
    const int nt = choose_nt(n, E);
    const int nt_g = exact_nt(nt, w->gu.fmt);
    // a rounded group-32 down projection reads an fp16 copy of the middle codes
    const int dfmt = down_fmt(w->dn.fmt, w->exact_down);
    const bool hd = dfmt == kFmtW4G32H;
    const int nt_d = exact_nt(nt, dfmt);
    {
        const int rc = run_gate_up(ws, w, n, nt_g, hd, s, mark);
        if (rc) return rc;
    }
    GemmArgs d = gemm_args(ws, w->dn, ws->s_m, ws->offsets, E, n, ws->y, H);
    if (launch_gemm(hd ? ws->map_qm_h[nt_index(nt_d)] : ws->map_qm[nt_index(nt_d)], d, dfmt,
                    kEpiStore, nt_d, ws->num_sms, s))
        return MOE_B200_ERR_UNSUPPORTED;
    mark(6);
    if (w->shared) {
        int rc = run_shared(ws, w, rows, d_x, s);
        if (rc) return rc;
    }
    mark(7);
    if (res_ready) cudaStreamWaitEvent(s, res_ready, 0);  // residual uploaded on the side
    launch_combine(ws->y, ws->pos, d_routes, w->shared ? ws->s_y : nullptr, d_res, rows, H, k,
                   d_out, s, gate.logits, gate.ld);
    mark(8);
    ws->last_rows = rows;
    ws->last_nt_gu = nt_g;
    ws->last_nt_dn = nt_d;
    ws->last_w = w;
    ws->last_stream = s;
    cudaError_t e = cudaPeekAtLastError();
    return cuda_rc(e);
}

float ev_ms(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, a, b);
    return ms;
}

void fill_timings_from(const cudaEvent_t* ev, moe_b200_workspace* ws, moe_b200_timings* t,
                       int rows, bool routed_by_us, bool shared) {
    memset(t, 0, sizeof(*t));
    t->router_us = routed_by_us ? 1000.0 * ev_ms(ev[0], ev[1]) : 0.0;
    t->schedule_us = 1000.0 * ev_ms(ev[1], ev[2]);
    t->input_us = 1000.0 * ev_ms(ev[2], ev[3]);
    t->gather_us = 0.0;  // the gather is fused into the input quantisation
    t->gate_us = 1000.0 * ev_ms(ev[3], ev[4]);
    t->middle_cpu_us = 1000.0 * ev_ms(ev[4], ev[5]);
    t->down_us = 1000.0 * ev_ms(ev[5], ev[6]);
    t->build_us = shared ? 1000.0 * ev_ms(ev[6], ev[7]) : 0.0;
    t->combine_us = 1000.0 * ev_ms(ev[7], ev[8]);
    t->total_us = 1000.0 * ev_ms(ev[0], ev[8]);
    t->gather_tasks = (int64_t)rows * ws->k;
    t->middle_tasks = (int64_t)rows * ws->k;
    t->gemm_tasks = 2;
}

void fill_timings(moe_b200_workspace* ws, moe_b200_timings* t, int rows, bool routed_by_us,
                  bool shared) {
    fill_timings_from(ws->ev, ws, t, rows, routed_by_us, shared);
}

int handle_status(moe_b200_workspace* ws, uint32_t bits, cudaStream_t s);

int read_status(moe_b200_workspace* ws, cudaStream_t s) {
    uint32_t bits = 0;
    cudaError_t e = cudaMemcpyAsync(&bits, ws->err, sizeof(bits), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_rc(e);
    return handle_status(ws, bits, s);
}

// The status bits of a finished call: cleared on the device, the counters a
// timed-out wait can leave mid-count rearmed, the first cause reported.
int handle_status(moe_b200_workspace* ws, uint32_t bits, cudaStream_t s) {
    if (bits) {
        cudaMemsetAsync(ws->err, 0, sizeof(uint32_t), s);
        // a wait that gave up can leave the grid barrier and the last-arrival
        // counters mid-count (CTAs that gave up never arrive): rearm them all,
        // so that no later call hands off early
        if (bits & kErrWaitTimeout) {
            const long T = ws->max_rows, n = ws->n_max;
            cudaMemsetAsync(ws->dec_bar, 0, sizeof(unsigned long long) * 128, s);
            cudaMemsetAsync(ws->w8r_acc, 0, sizeof(int32_t) * ws->w8r_acc_n, s);
            cudaMemsetAsync(ws->w8r_cnt, 0, sizeof(int) * ws->w8r_cnt_n, s);
            cudaMemsetAsync(ws->w8r_max, 0, sizeof(uint32_t) * (size_t)kGemvMaxRows * ws->k, s);
            cudaMemsetAsync(ws->gv_counters, 0, sizeof(int) * (size_t)(n + T * ((ws->H + 127) / 128)), s);
            cudaMemsetAsync(ws->counters, 0, sizeof(int) * (size_t)T, s);
            if (ws->Is > 0) {
                cudaMemsetAsync(ws->w8_acc, 0, sizeof(int32_t) * (size_t)kGemvMaxRows *
                                    std::max(2L * pad_to(ws->Is, 64), (long)pad_to(ws->H, 128)), s);
                cudaMemsetAsync(ws->w8_cnt, 0, sizeof(int) * 1024, s);
                cudaMemsetAsync(ws->w8_max, 0, sizeof(uint32_t) * kGemvMaxRows, s);
            }

        }
        cudaStreamSynchronize(s);
    }
    return map_err_bits(bits);
}

int validate_host_routes(const moe_b200_workspace* ws, int rows, const int32_t* ids,
                         const float* routes) {
    const long n = (long)rows * ws->k;
    for (long a = 0; a < n; ++a) {
        if (!(routes[a] >= 0.0f) || !(routes[a] <= 3.4e38f)) return MOE_B200_ERR_BAD_ROUTE;
        if (routes[a] > 0.0f && (ids[a] < 0 || ids[a] >= ws->E)) return MOE_B200_ERR_BAD_EXPERT;
    }
    return MOE_B200_OK;
}

}  // namespace

// ===================================================================== C ABI

extern "C" {

void moe_b200_config_init(moe_b200_config* cfg, int32_t hidden, int32_t intermediate,
                          int32_t experts, int32_t shared, int32_t top, int32_t max_rows) {
    if (!cfg) return;
    memset(cfg, 0, sizeof(*cfg));
    cfg->weights.hidden = hidden;
    cfg->weights.intermediate = intermediate;
    cfg->weights.routed_experts = experts;
    cfg->weights.shared_expert = shared ? 1 : 0;
    cfg->weights.shared_intermediate = 0;
    cfg->top = top;
    cfg->max_rows = max_rows;
    cfg->device = 0;
    cfg->npu_cores = 0;
    cfg->cpu_threads = 0;
}

static int validate_config(const moe_b200_config* cfg) {
    if (!cfg) return MOE_B200_ERR_INVALID;
    const moe_b200_weight_config& w = cfg->weights;
    if (w.hidden <= 0 || w.intermediate <= 0 || w.routed_experts <= 0 || cfg->top <= 0 ||
        cfg->max_rows <= 0)
        return MOE_B200_ERR_INVALID;
    if (cfg->top > w.routed_experts || cfg->top > 32 || w.routed_experts > 1024)
        return MOE_B200_ERR_UNSUPPORTED;
    if (w.hidden % 32 || w.intermediate % 32) return MOE_B200_ERR_UNSUPPORTED;
    const int is = w.shared_intermediate > 0 ? w.shared_intermediate : w.intermediate;
    if (w.shared_expert && is % 32) return MOE_B200_ERR_UNSUPPORTED;
    return MOE_B200_OK;
}

moe_b200_weights* moe_b200_weights_create(const moe_b200_config* cfg,
                                          const moe_b200_expert* experts,
                                          const moe_b200_format* format) {
    if (validate_config(cfg) || !experts) return nullptr;
    if (check_device(cfg->device, nullptr)) return nullptr;
    DeviceGuard guard(cfg->device);
    moe_b200_format fmt{MOE_B200_W4_PER_CHANNEL, MOE_B200_W8_PER_CHANNEL, MOE_B200_SHARED_JOINT};
    if (format) fmt = *format;
    const int H = cfg->weights.hidden, I = cfg->weights.intermediate, E = cfg->weights.routed_experts;
    const int Is = cfg->weights.shared_intermediate > 0 ? cfg->weights.shared_intermediate : I;
    if (fmt.routed_format < 0 || fmt.routed_format > MOE_B200_W4_G32_FP16_ROUNDED_DOWN) return nullptr;
    const bool exact_down = fmt.routed_format != MOE_B200_W4_G32_FP16_ROUNDED_DOWN;
    if (fmt.routed_format == MOE_B200_W4_G32_FP16_EXACT ||
        fmt.routed_format == MOE_B200_W4_G32_FP16_ROUNDED_DOWN)
        fmt.routed_format = MOE_B200_W4_G32_FP16;  // one packing for all three
    if (fmt.shared_format != MOE_B200_W8_PER_CHANNEL && fmt.shared_format != MOE_B200_W4_PER_CHANNEL)
        return nullptr;
    if (cfg->weights.shared_expert && fmt.shared_mode == MOE_B200_SHARED_JOINT && Is != I)
        return nullptr;  // joint bank needs the routed intermediate (src/npu/moe.rs:230-233)
    for (int e = 0; e < E + (cfg->weights.shared_expert ? 1 : 0); ++e) {
        const moe_b200_expert& x = experts[e];
        const int f = e < E ? fmt.routed_format : fmt.shared_format;
        if (!x.gate_up || !x.down) return nullptr;
        if (f == MOE_B200_W4_G32_FP16 && (!x.gate_up_group_scales || !x.down_group_scales))
            return nullptr;
        if (f != MOE_B200_W4_G32_FP16 && (!x.gate_up_scales || !x.down_scales)) return nullptr;
    }

    auto* w = new moe_b200_weights();
    w->device = cfg->device;
    w->H = H;
    w->I = I;
    w->E = E;
    w->top = cfg->top;
    w->shared = cfg->weights.shared_expert;
    w->Is = Is;
    w->shared_mode = fmt.shared_mode;
    w->exact_down = exact_down;
    setup_mat(w->gu, fmt.routed_format, E, H, I, true);
    setup_mat(w->dn, fmt.routed_format, E, I, H, false);
    if (w->shared) {
        setup_mat(w->sgu, fmt.shared_format, 1, H, Is, true);
        setup_mat(w->sdn, fmt.shared_format, 1, Is, H, false);
    }
    bool ok = true;
    auto build = [&](PackedMat& m, int first, int count) {
        const size_t wb = m.w_expert_stride * count, sb = m.s_expert_stride * count;
        std::vector<uint8_t> hw(wb, 0), hs(sb, 0);
        for (int e = 0; e < count; ++e) {
            const moe_b200_expert& x = experts[first + e];
            const bool is_gu = m.swiglu;
            pack_expert(m, is_gu ? x.gate_up : x.down, is_gu ? x.gate_up_scales : x.down_scales,
                        is_gu ? x.gate_up_group_scales : x.down_group_scales,
                        hw.data() + m.w_expert_stride * e, hs.data() + m.s_expert_stride * e);
        }
        void *dw = nullptr, *ds = nullptr;
        if (dev_alloc(&dw, wb) != cudaSuccess) { ok = false; return; }
        if (dev_alloc(&ds, sb) != cudaSuccess) { cudaFree(dw); ok = false; return; }
        m.w = static_cast<uint8_t*>(dw);
        m.s = ds;
        if (cudaMemcpy(dw, hw.data(), wb, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(ds, hs.data(), sb, cudaMemcpyHostToDevice) != cudaSuccess)
            ok = false;
        w->bytes += wb + sb;
    };
    build(w->gu, 0, E);
    if (ok) build(w->dn, 0, E);
    if (ok && w->shared) build(w->sgu, E, 1);
    if (ok && w->shared) build(w->sdn, E, 1);
    if (!ok) {
        moe_b200_weights_free(w);
        return nullptr;
    }
    return w;
}

void moe_b200_weights_free(moe_b200_weights* w) {
    if (!w) return;
    DeviceGuard guard(w->device);
    for (PackedMat* m : {&w->gu, &w->dn, &w->sgu, &w->sdn}) {
        if (m->w) cudaFree(m->w);
        if (m->s) cudaFree(m->s);
    }
    delete w;
}

uint64_t moe_b200_weights_device_bytes(const moe_b200_weights* w) { return w ? w->bytes : 0; }

// ---- expert slot bank -------------------------------------------------------
// A blob is one routed expert's packed device image: a 64-byte header, then
// the gate|up weights, their scales, the down weights and their scales, each
// exactly as they sit in the bank (tile-major, swizzled), so import and export
// are plain copies.

namespace {

constexpr char kBlobMagic[8] = {'M', 'B', '2', 'X', 'B', 'L', 'O', 'B'};

struct BlobHeader {
    char magic[8];
    uint32_t version, format, hidden, intermediate;
    uint64_t sizes[4];  // gate|up weights, gate|up scales, down weights, down scales
    uint8_t pad[8];
};
static_assert(sizeof(BlobHeader) == 64, "blob header is 64 bytes");

struct Region {
    uint8_t* dev;
    uint64_t bytes;
};

// The four device regions of expert e (weights of group-32 banks carry their
// scales inside; their scale regions hold the unused per-channel slots).
void expert_regions(const moe_b200_weights* w, int e, Region r[4]) {
    r[0] = {w->gu.w + w->gu.w_expert_stride * e, w->gu.w_expert_stride};
    r[1] = {static_cast<uint8_t*>(w->gu.s) + w->gu.s_expert_stride * e, w->gu.s_expert_stride};
    r[2] = {w->dn.w + w->dn.w_expert_stride * e, w->dn.w_expert_stride};
    r[3] = {static_cast<uint8_t*>(w->dn.s) + w->dn.s_expert_stride * e, w->dn.s_expert_stride};
}

uint32_t public_format(const moe_b200_weights* w) {
    if (w->gu.fmt == kFmtW4G32)
        return w->exact_down ? MOE_B200_W4_G32_FP16 : MOE_B200_W4_G32_FP16_ROUNDED_DOWN;
    return (uint32_t)w->gu.fmt;  // kFmtW4PC / kFmtW8PC match the public values
}

BlobHeader blob_header(const moe_b200_weights* w) {
    BlobHeader h{};
    std::memcpy(h.magic, kBlobMagic, 8);
    h.version = MOE_B200_BLOB_VERSION;
    h.format = public_format(w);
    h.hidden = (uint32_t)w->H;
    h.intermediate = (uint32_t)w->I;
    Region r[4];
    expert_regions(w, 0, r);
    for (int i = 0; i < 4; ++i) h.sizes[i] = r[i].bytes;
    return h;
}

uint64_t blob_size(const moe_b200_weights* w) {
    const BlobHeader h = blob_header(w);
    return sizeof(BlobHeader) + h.sizes[0] + h.sizes[1] + h.sizes[2] + h.sizes[3];
}

int check_blob(const moe_b200_weights* w, const void* data, uint64_t bytes) {
    if (!data || bytes != blob_size(w)) return MOE_B200_ERR_INVALID;
    BlobHeader got;
    std::memcpy(&got, data, sizeof(got));
    const BlobHeader want = blob_header(w);
    if (std::memcmp(got.magic, want.magic, 8) || got.version != want.version ||
        got.format != want.format || got.hidden != want.hidden ||
        got.intermediate != want.intermediate || std::memcmp(got.sizes, want.sizes, sizeof(got.sizes)))
        return MOE_B200_ERR_INVALID;
    return MOE_B200_OK;
}

}  // namespace

uint32_t moe_b200_blob_version(void) { return MOE_B200_BLOB_VERSION; }

moe_b200_weights* moe_b200_slots_create(const moe_b200_config* cfg, int32_t routed_format) {
    if (validate_config(cfg) || cfg->weights.shared_expert) return nullptr;
    if (routed_format < 0 || routed_format > MOE_B200_W4_G32_FP16_ROUNDED_DOWN) return nullptr;
    if (check_device(cfg->device, nullptr)) return nullptr;
    DeviceGuard guard(cfg->device);
    const bool exact_down = routed_format != MOE_B200_W4_G32_FP16_ROUNDED_DOWN;
    const int f = (routed_format == MOE_B200_W4_G32_FP16_EXACT ||
                   routed_format == MOE_B200_W4_G32_FP16_ROUNDED_DOWN)
                      ? MOE_B200_W4_G32_FP16
                      : routed_format;
    auto* w = new moe_b200_weights();
    w->device = cfg->device;
    w->H = cfg->weights.hidden;
    w->I = cfg->weights.intermediate;
    w->E = cfg->weights.routed_experts;
    w->top = cfg->top;
    w->Is = w->I;
    w->exact_down = exact_down;
    setup_mat(w->gu, f, w->E, w->H, w->I, true);
    setup_mat(w->dn, f, w->E, w->I, w->H, false);
    for (PackedMat* m : {&w->gu, &w->dn}) {
        const size_t wb = m->w_expert_stride * w->E, sb = m->s_expert_stride * w->E;
        void *dw = nullptr, *ds = nullptr;
        if (dev_alloc(&dw, wb) != cudaSuccess || dev_alloc(&ds, sb) != cudaSuccess ||
            cudaMemset(dw, 0, wb) != cudaSuccess || cudaMemset(ds, 0, sb) != cudaSuccess) {
            if (dw) cudaFree(dw);
            if (ds) cudaFree(ds);
            moe_b200_weights_free(w);
            return nullptr;
        }
        m->w = static_cast<uint8_t*>(dw);
        m->s = ds;
        w->bytes += wb + sb;
    }
    return w;
}

uint64_t moe_b200_expert_blob_bytes(const moe_b200_weights* w) { return w ? blob_size(w) : 0; }

int moe_b200_export_expert(const moe_b200_weights* w, int32_t expert, void* data, uint64_t bytes) {
    if (!w || !data || bytes != blob_size(w)) return MOE_B200_ERR_INVALID;
    if (expert < 0 || expert >= w->E) return MOE_B200_ERR_BAD_EXPERT;
    DeviceGuard guard(w->device);
    const BlobHeader h = blob_header(w);
    std::memcpy(data, &h, sizeof(h));
    uint8_t* dst = static_cast<uint8_t*>(data) + sizeof(h);
    Region r[4];
    expert_regions(w, expert, r);
    for (const Region& g : r) {
        const cudaError_t e = cudaMemcpy(dst, g.dev, g.bytes, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_rc(e);
        dst += g.bytes;
    }
    return MOE_B200_OK;
}

int moe_b200_import_expert_async(moe_b200_weights* w, int32_t slot, const void* data,
                                 uint64_t bytes, void* stream) {
    if (!w) return MOE_B200_ERR_INVALID;
    int rc = check_blob(w, data, bytes);
    if (rc) return rc;
    if (slot < 0 || slot >= w->E) return MOE_B200_ERR_BAD_EXPERT;
    DeviceGuard guard(w->device);
    const uint8_t* src = static_cast<const uint8_t*>(data) + sizeof(BlobHeader);
    Region r[4];
    expert_regions(w, slot, r);
    for (const Region& g : r) {
        const cudaError_t e = cudaMemcpyAsync(g.dev, src, g.bytes, cudaMemcpyHostToDevice,
                                              static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_rc(e);
        src += g.bytes;
    }
    return MOE_B200_OK;
}

int moe_b200_import_expert(moe_b200_weights* w, int32_t slot, const void* data, uint64_t bytes) {
    int rc = moe_b200_import_expert_async(w, slot, data, bytes, nullptr);
    if (rc) return rc;
    DeviceGuard guard(w->device);
    return cuda_rc(cudaStreamSynchronize(nullptr));
}

int moe_b200_swap_slots(moe_b200_weights* bank, int32_t slot, moe_b200_weights* staging,
                        int32_t staged, void* stream) {
    if (!bank || !staging || bank->device != staging->device) return MOE_B200_ERR_INVALID;
    if (blob_size(bank) != blob_size(staging) || public_format(bank) != public_format(staging) ||
        bank->H != staging->H || bank->I != staging->I)
        return MOE_B200_ERR_INVALID;
    if (slot < 0 || slot >= bank->E || staged < 0 || staged >= staging->E)
        return MOE_B200_ERR_BAD_EXPERT;
    if (bank == staging && slot == staged) return MOE_B200_OK;
    DeviceGuard guard(bank->device);
    Region a[4], b[4];
    expert_regions(bank, slot, a);
    expert_regions(staging, staged, b);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < 4; ++i) launch_swap_bytes(a[i].dev, b[i].dev, a[i].bytes, s);
    return cuda_rc(cudaPeekAtLastError());
}

moe_b200_workspace* moe_b200_workspace_create(const moe_b200_config* cfg) {
    if (validate_config(cfg)) return nullptr;
    int sms = 0;
    if (check_device(cfg->device, &sms)) return nullptr;
    DeviceGuard guard(cfg->device);
    auto* ws = new moe_b200_workspace();
    ws->device = cfg->device;
    ws->H = cfg->weights.hidden;
    ws->I = cfg->weights.intermediate;
    ws->E = cfg->weights.routed_experts;
    ws->k = cfg->top;
    ws->max_rows = cfg->max_rows;
    ws->Is = cfg->weights.shared_expert
                 ? (cfg->weights.shared_intermediate > 0 ? cfg->weights.shared_intermediate : ws->I)
                 : 0;
    ws->num_sms = sms;
    ws->Kh = pad_to(ws->H, kKAlign);
    ws->Ki = pad_to(ws->I, kKAlign);
    ws->Kis = pad_to(ws->Is > 0 ? ws->Is : 32, kKAlign);
    const long T = ws->max_rows, n = T * ws->k;
    ws->n_max = n;
    const long nb = (n + kRouteChunk - 1) / kRouteChunk;
    const long pad_rows = 64;  // tiles may read past the last row
    int rc = MOE_B200_OK;
    rc |= ws_alloc(ws, &ws->x, T * ws->H);
    rc |= ws_alloc(ws, &ws->out, T * ws->H);
    rc |= ws_alloc(ws, &ws->res, T * ws->H);
    rc |= ws_alloc(ws, &ws->routes, n);
    rc |= ws_alloc(ws, &ws->ids, n);
    rc |= ws_alloc(ws, &ws->q_x, (T + pad_rows) * ws->Kh);
    rc |= ws_alloc(ws, &ws->s_x, T);
    rc |= ws_alloc(ws, &ws->hist, (nb > 0 ? nb : 1) * ws->E);
    rc |= ws_alloc(ws, &ws->offsets, ws->E + 1);
    rc |= ws_alloc(ws, &ws->perm, n);
    rc |= ws_alloc(ws, &ws->pos, n);
    rc |= ws_alloc(ws, &ws->shared_offsets, 2);
    rc |= ws_alloc(ws, &ws->counters, T);
    rc |= ws_alloc(ws, &ws->gv_counters, n + T * ((ws->H + 127) / 128));
    rc |= ws_alloc(ws, &ws->dec_state, 2 * n + 2);
    rc |= ws_alloc(ws, &ws->dec_bar, 128);
    {
        const long ns = (long)kGemvMaxRows * ws->k;
        const long gt = (ws->I + 63) / 64, dt = (ws->H + 127) / 128;
        ws->w8r_acc_n = (size_t)ns * std::max(gt, dt) * 128;
        ws->w8r_cnt_n = (size_t)(ns * gt + ns + ns * dt + (long)kGemvMaxRows * dt);
        rc |= ws_alloc(ws, &ws->w8r_acc, (long)ws->w8r_acc_n);
        rc |= ws_alloc(ws, &ws->w8r_cnt, (long)ws->w8r_cnt_n);
        rc |= ws_alloc(ws, &ws->w8r_max, ns);
    }
    rc |= ws_alloc(ws, &ws->a_perm, (n + pad_rows) * ws->Kh);
    rc |= ws_alloc(ws, &ws->q_m_h, (n + pad_rows) * ws->Ki);
    rc |= ws_alloc(ws, &ws->s_perm, n);
    rc |= ws_alloc(ws, &ws->gate_up, n * 2 * ws->I);
    rc |= ws_alloc(ws, &ws->q_m, (n + pad_rows) * ws->Ki);
    rc |= ws_alloc(ws, &ws->s_m, n);
    rc |= ws_alloc(ws, &ws->y, n * ws->H);

    rc |= ws_alloc(ws, &ws->logits, T * (ws->E + 1));  // + the shared-gate column
    rc |= ws_alloc(ws, &ws->err, 1);
    if (ws->Is > 0 && rc == MOE_B200_OK) {
        rc |= ws_alloc(ws, &ws->q_xd, (T + pad_rows) * ws->Kh);
        rc |= ws_alloc(ws, &ws->s_xd, T);
        rc |= ws_alloc(ws, &ws->s_middle, T * 2 * ws->Is);
        rc |= ws_alloc(ws, &ws->sq_m, (T + pad_rows) * ws->Kis);
        rc |= ws_alloc(ws, &ws->sq_m_h, (T + pad_rows) * ws->Kis);
        rc |= ws_alloc(ws, &ws->ss_m, T);
        rc |= ws_alloc(ws, &ws->s_y, T * ws->H);
        rc |= ws_alloc(ws, &ws->w8_acc, (long)kGemvMaxRows * std::max(2L * pad_to(ws->Is, 64),
                                                                      (long)pad_to(ws->H, 128)));
        rc |= ws_alloc(ws, &ws->w8_cnt, 1024);
        rc |= ws_alloc(ws, &ws->w8_max, kGemvMaxRows);
    }
    if (rc != MOE_B200_OK) {
        moe_b200_workspace_free(ws);
        return nullptr;
    }
    cudaMemset(ws->counters, 0, sizeof(int) * T);
    cudaMemset(ws->gv_counters, 0, sizeof(int) * (size_t)(n + T * ((ws->H + 127) / 128)));
    cudaMemset(ws->dec_state, 0, sizeof(uint32_t) * (size_t)(2 * n + 2));
    cudaMemset(ws->dec_bar, 0, sizeof(unsigned long long) * 128);
    cudaMemset(ws->w8r_acc, 0, sizeof(int32_t) * ws->w8r_acc_n);
    cudaMemset(ws->w8r_cnt, 0, sizeof(int) * ws->w8r_cnt_n);
    cudaMemset(ws->w8r_max, 0, sizeof(uint32_t) * (size_t)kGemvMaxRows * ws->k);
    if (ws->Is > 0) {
        cudaMemset(ws->w8_acc, 0, sizeof(int32_t) * (size_t)kGemvMaxRows *
                                      std::max(2L * pad_to(ws->Is, 64), (long)pad_to(ws->H, 128)));
        cudaMemset(ws->w8_cnt, 0, sizeof(int) * 1024);
        cudaMemset(ws->w8_max, 0, sizeof(uint32_t) * kGemvMaxRows);
    }

    {
        int coop = 0;
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ws->device);
        ws->coop = coop != 0;
    }
    cudaMemset(ws->err, 0, sizeof(uint32_t));
    cudaMemset(ws->a_perm, 0, (size_t)(n + pad_rows) * ws->Kh);
    cudaMemset(ws->q_m, 0, (size_t)(n + pad_rows) * ws->Ki);
    cudaMemset(ws->q_x, 0, (size_t)(T + pad_rows) * ws->Kh);
    cudaMemset(ws->q_m_h, 0, sizeof(__half) * (size_t)(n + pad_rows) * ws->Ki);
    for (int i = 0; i < 3 && rc == MOE_B200_OK; ++i) {
        const int nt = kNTs[i];
        rc |= make_act_map(&ws->map_a[i], ws->a_perm, (int)(n + pad_rows), ws->Kh, nt);
        rc |= make_act_map(&ws->map_qm[i], ws->q_m, (int)(n + pad_rows), ws->Ki, nt);
        rc |= make_act_map(&ws->map_qx[i], ws->q_x, (int)(T + pad_rows), ws->Kh, nt);
        rc |= make_act_map_h(&ws->map_qm_h[i], ws->q_m_h, (int)(n + pad_rows), ws->Ki, nt);
        if (ws->Is > 0) {
            rc |= make_act_map(&ws->map_qxd[i], ws->q_xd, (int)(T + pad_rows), ws->Kh, nt);
            rc |= make_act_map(&ws->map_sqm[i], ws->sq_m, (int)(T + pad_rows), ws->Kis, nt);
            rc |= make_act_map_h(&ws->map_sqm_h[i], ws->sq_m_h, (int)(T + pad_rows), ws->Kis, nt);
        }
    }
    if (rc == MOE_B200_OK &&
        (cudaStreamCreateWithFlags(&ws->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
         cudaStreamCreateWithFlags(&ws->side_stream, cudaStreamNonBlocking) != cudaSuccess ||
         cudaEventCreateWithFlags(&ws->side_fork, cudaEventDisableTiming) != cudaSuccess ||
         cudaEventCreateWithFlags(&ws->side_join, cudaEventDisableTiming) != cudaSuccess ||
         cudaMallocHost(&ws->h_err, sizeof(uint32_t)) != cudaSuccess ||
         cudaEventCreateWithFlags(&ws->res_ready, cudaEventDisableTiming) != cudaSuccess ||
         cudaEventCreateWithFlags(&ws->x_ready, cudaEventDisableTiming) != cudaSuccess))
        rc = MOE_B200_ERR_CUDA;
    if (rc == MOE_B200_OK && cudaStreamCreateWithFlags(&ws->own_stream, cudaStreamNonBlocking) != cudaSuccess)
        rc = MOE_B200_ERR_CUDA;

    for (int i = 0; i < 12 && rc == MOE_B200_OK; ++i)
        if (cudaEventCreate(&ws->ev[i]) != cudaSuccess) rc = MOE_B200_ERR_CUDA;
    if (rc != MOE_B200_OK || cudaDeviceSynchronize() != cudaSuccess) {
        moe_b200_workspace_free(ws);
        return nullptr;
    }
    return ws;
}

void moe_b200_workspace_free(moe_b200_workspace* ws) {
    if (!ws) return;
    DeviceGuard guard(ws->device);
    if (ws->own_stream) cudaStreamSynchronize(ws->own_stream);
    for (void* p : ws->allocs) cudaFree(p);
    for (int i = 0; i < 12; ++i)
        if (ws->ev[i]) cudaEventDestroy(ws->ev[i]);
    for (cudaEvent_t e : ws->prof_ev) cudaEventDestroy(e);
    if (ws->own_stream) cudaStreamDestroy(ws->own_stream);
    if (ws->side_stream) {
        cudaStreamSynchronize(ws->side_stream);
        cudaStreamDestroy(ws->side_stream);
    }
    if (ws->side_fork) cudaEventDestroy(ws->side_fork);
    if (ws->h_err) cudaFreeHost(ws->h_err);
    if (ws->hg.exec) cudaGraphExecDestroy(ws->hg.exec);
    if (ws->hg.graph) cudaGraphDestroy(ws->hg.graph);
    if (ws->side_join) cudaEventDestroy(ws->side_join);
    if (ws->copy_stream) {
        cudaStreamSynchronize(ws->copy_stream);
        cudaStreamDestroy(ws->copy_stream);
    }
    if (ws->res_ready) cudaEventDestroy(ws->res_ready);
    if (ws->x_ready) cudaEventDestroy(ws->x_ready);
    delete ws;
}

uint64_t moe_b200_workspace_device_bytes(const moe_b200_workspace* ws) { return ws ? ws->bytes : 0; }

int32_t moe_b200_max_rows(const moe_b200_workspace* ws) { return ws ? ws->max_rows : 0; }

int moe_b200_run_device(moe_b200_workspace* ws, const moe_b200_weights* w, int32_t rows,
                        const float* d_input, const int32_t* d_ids, const float* d_routes,
                        float* d_output, void* stream) {
    int rc = compatible(ws, w);
    if (rc) return rc;
    if (rows < 0) return MOE_B200_ERR_INVALID;
    if (rows > ws->max_rows) return MOE_B200_ERR_CAPACITY;
    if (rows == 0) return MOE_B200_OK;
    if (!d_input || !d_ids || !d_routes || !d_output) return MOE_B200_ERR_INVALID;
    if (!aligned16(d_input) || !aligned16(d_output)) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaEvent_t* evs = prof_slot(ws, w->shared ? 2 : 0);
    if (evs) {
        cudaEventRecord(evs[0], s);
        cudaEventRecord(evs[1], s);
    }
    return run_pipeline(ws, w, rows, d_input, d_ids, d_routes, nullptr, d_output, s, evs);
}

int moe_b200_run_f32(moe_b200_workspace* ws, const moe_b200_weights* w, int32_t rows,
                     const float* input, const int32_t* ids, const float* routes, float* output,
                     moe_b200_timings* timings) {
    int rc = compatible(ws, w);
    if (rc) return rc;
    if (rows < 0) return MOE_B200_ERR_INVALID;
    if (rows > ws->max_rows) return MOE_B200_ERR_CAPACITY;
    if (rows == 0) return MOE_B200_OK;
    if (!input || !ids || !routes || !output) return MOE_B200_ERR_INVALID;
    rc = validate_host_routes(ws, rows, ids, routes);
    if (rc) return rc;
    DeviceGuard guard(ws->device);
    cudaStream_t s = ws->own_stream;
    const size_t xb = sizeof(float) * (size_t)rows * ws->H, nb = (size_t)rows * ws->k;
    if (timings) cudaEventRecord(ws->ev[0], s);
    cudaMemcpyAsync(ws->x, input, xb, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(ws->ids, ids, sizeof(int32_t) * nb, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(ws->routes, routes, sizeof(float) * nb, cudaMemcpyHostToDevice, s);
    rc = run_pipeline(ws, w, rows, ws->x, ws->ids, ws->routes, nullptr, ws->out, s,
                      timings ? ws->ev : nullptr);
    if (rc) return rc;
    cudaMemcpyAsync(output, ws->out, xb, cudaMemcpyDeviceToHost, s);
    if (timings) cudaEventRecord(ws->ev[9], s);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_rc(e);
    rc = read_status(ws, s);
    if (timings) {
        fill_timings(ws, timings, rows, false, w->shared != 0);
        timings->sync_us = 1000.0 * ev_ms(ws->ev[8], ws->ev[9]);
        timings->total_us = 1000.0 * ev_ms(ws->ev[0], ws->ev[9]);
    }
    return rc;
}

void moe_b200_router_options_init(moe_b200_router_options* opt) {
    if (!opt) return;
    *opt = moe_b200_router_options{};
    opt->order = MOE_B200_ROUTER_NEON16;
    opt->rule = MOE_B200_ROUTE_SOFTMAX;
    opt->groups = 1;
    opt->top_groups = 1;
    opt->routing_scale = 1.0f;
}

static bool finite_all(const float* v, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(v[i])) return false;
    return true;
}

moe_b200_router* moe_b200_router_create_ex(const moe_b200_config* cfg, const float* router,
                                           const moe_b200_router_options* opt) {
    if (validate_config(cfg) || !router || !opt) return nullptr;
    const int H = cfg->weights.hidden, E = cfg->weights.routed_experts, k = cfg->top;
    if (opt->order != MOE_B200_ROUTER_NEON16 && opt->order != MOE_B200_ROUTER_SEQUENTIAL &&
        opt->order != MOE_B200_ROUTER_TF32)
        return nullptr;
    if (!(opt->min_weight >= 0.0f && opt->min_weight <= 1.0f)) return nullptr;  // pruning::validate
    if (opt->rule == MOE_B200_ROUTE_GROUPED_SIGMOID) {
        // the Ling config check (src/model/ling3tiny/config.rs:113-124) plus
        // this kernel's limits (one warp per row: E <= 256, groups <= 32)
        const int g = opt->groups, tg = opt->top_groups;
        if (g <= 0 || g > 32 || E % g != 0 || E / g < 2 || tg <= 0 || tg > g ||
            k > tg * (E / g) || !(opt->routing_scale > 0.0f) || !opt->expert_bias ||
            E > moe::kGroupedMaxExperts || opt->min_weight != 0.0f)
            return nullptr;
        if (!finite_all(opt->expert_bias, (size_t)E)) return nullptr;
    } else if (opt->rule != MOE_B200_ROUTE_SOFTMAX) {
        return nullptr;
    }
    if (check_device(cfg->device, nullptr)) return nullptr;
    DeviceGuard guard(cfg->device);
    auto* r = new moe_b200_router();
    r->device = cfg->device;
    r->H = H;
    r->E = E;
    r->order = opt->order;
    r->min_weight = opt->min_weight;
    r->rule = opt->rule;
    r->groups = opt->groups;
    r->top_groups = opt->top_groups;
    r->scale = opt->routing_scale;
    r->gate = opt->shared_gate != nullptr;
    const size_t row_bytes = sizeof(float) * (size_t)H;
    void* p = nullptr;
    if (dev_alloc(&p, row_bytes * r->rows()) != cudaSuccess) { delete r; return nullptr; }
    r->w = static_cast<float*>(p);
    if (opt->order == MOE_B200_ROUTER_TF32) {
        // the NPU narrows the resident weights once (src/npu/tf32.rs:114-140)
        std::vector<float> t((size_t)H * r->rows());
        std::memcpy(t.data(), router, row_bytes * E);
        if (r->gate) std::memcpy(t.data() + (size_t)E * H, opt->shared_gate, row_bytes);
        for (float& v : t) {
            uint32_t u;
            std::memcpy(&u, &v, 4);
            u &= ~0x1FFFu;
            std::memcpy(&v, &u, 4);
        }
        cudaMemcpy(r->w, t.data(), row_bytes * r->rows(), cudaMemcpyHostToDevice);
    } else {
        cudaMemcpy(r->w, router, row_bytes * E, cudaMemcpyHostToDevice);
        if (r->gate)
            cudaMemcpy(r->w + (size_t)E * H, opt->shared_gate, row_bytes, cudaMemcpyHostToDevice);
    }
    auto upload = [&](float** dst, const float* src) {
        if (!src) return true;
        void* q = nullptr;
        if (dev_alloc(&q, sizeof(float) * E) != cudaSuccess) return false;
        *dst = static_cast<float*>(q);
        return cudaMemcpy(*dst, src, sizeof(float) * E, cudaMemcpyHostToDevice) == cudaSuccess;
    };
    if (!upload(&r->bias, opt->bias) ||
        !upload(&r->sel_bias, opt->rule == MOE_B200_ROUTE_GROUPED_SIGMOID ? opt->expert_bias
                                                                         : nullptr)) {
        moe_b200_router_free(r);
        return nullptr;
    }
    return r;
}

moe_b200_router* moe_b200_router_create(const moe_b200_config* cfg, const float* router,
                                        const float* bias, int32_t order, float min_weight) {
    moe_b200_router_options opt;
    moe_b200_router_options_init(&opt);
    opt.order = order;
    opt.min_weight = min_weight;
    opt.bias = bias;
    return moe_b200_router_create_ex(cfg, router, &opt);
}

void moe_b200_router_free(moe_b200_router* r) {
    if (!r) return;
    DeviceGuard guard(r->device);
    if (r->w) cudaFree(r->w);
    if (r->bias) cudaFree(r->bias);
    if (r->sel_bias) cudaFree(r->sel_bias);
    delete r;
}

static GateRef router_gate(const moe_b200_workspace* ws, const moe_b200_router* r) {
    GateRef g;
    if (r->gate) {
        g.logits = ws->logits + r->E;
        g.ld = r->rows();
    }
    return g;
}

static RouterArgs router_args(moe_b200_workspace* ws, const moe_b200_router* r, int rows,
                              const float* d_x, float* d_logits, int32_t* d_ids, float* d_routes) {
    RouterArgs a{};
    a.x = d_x;
    a.w = r->w;
    a.bias = r->bias;
    a.T = rows;
    a.H = r->H;
    a.E = r->E;
    a.Ew = r->rows();
    a.k = ws->k;
    a.order = r->order;
    a.min_weight = r->min_weight;
    a.rule = r->rule;
    a.sel_bias = r->sel_bias;
    a.groups = r->groups;
    a.top_groups = r->top_groups;
    a.scale = r->scale;
    a.logits = d_logits ? d_logits : ws->logits;
    a.counters = ws->counters;
    a.ids = d_ids;
    a.weights = d_routes;
    a.err = ws->err;
    return a;
}

static int route_impl(moe_b200_workspace* ws, const moe_b200_router* r, int rows, const float* d_x,
                      float* d_logits, int32_t* d_ids, float* d_routes, cudaStream_t s) {
    const RouterArgs a = router_args(ws, r, rows, d_x, d_logits, d_ids, d_routes);
    ws->last_logit_cols = r->rows();
    if (launch_router(a, s)) return MOE_B200_ERR_UNSUPPORTED;  // geometry does not fit
    // the decode-sized router routes in its last CTA; the others launch a
    // separate routing kernel
    ws->launches += (r->order == MOE_B200_ROUTER_SEQUENTIAL || rows >= 16) ? 2 : 1;
    return cuda_rc(cudaPeekAtLastError());
}

int moe_b200_route_device(moe_b200_workspace* ws, const moe_b200_router* r, int32_t rows,
                          const float* d_input, float* d_logits, int32_t* d_ids, float* d_routes,
                          void* stream) {
    if (!ws || !r || r->H != ws->H || r->E != ws->E || r->device != ws->device)
        return MOE_B200_ERR_INVALID;
    if (rows < 0) return MOE_B200_ERR_INVALID;
    if (rows > ws->max_rows) return MOE_B200_ERR_CAPACITY;
    if (rows == 0) return MOE_B200_OK;
    if (!d_input || !d_ids || !d_routes || !aligned16(d_input)) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ws->last_stream = s;
    return route_impl(ws, r, rows, d_input, d_logits, d_ids, d_routes, s);
}

// The router-inclusive layer: one cooperative launch of the fused small-batch
// kernel where it applies (group-32 bank without a shared expert, at most
// kFusedMaxRows tokens, NEON16 or TF32 router without a gate row), else the
// router followed by the pipeline. The fused kernel's time shows as the
// gate/up stage of the profiling events.
static int layer_impl(moe_b200_workspace* ws, const moe_b200_weights* w, const moe_b200_router* r,
                      int rows, const float* d_x, const float* d_res, float* d_out, cudaStream_t s,
                      cudaEvent_t* evs, cudaEvent_t res_ready) {
    if (ws->coop && rows <= kFusedMaxRows && use_gemv(ws, w, rows) && !w->shared &&
        r->order != MOE_B200_ROUTER_SEQUENTIAL && !r->gate) {
        if (res_ready) cudaStreamWaitEvent(s, res_ready, 0);
        DecodeArgs d{};
        d.r = router_args(ws, r, rows, d_x, nullptr, ws->ids, ws->routes);
        d.g = gemv_args(ws, w, rows, d_x, ws->ids, ws->routes, d_res, d_out);
        d.bar = ws->dec_bar;
        d.mmax = ws->dec_state + 2;
        d.ready = ws->dec_state + 2 + ws->n_max;
        for (int i = 1; evs && i <= 3; ++i) cudaEventRecord(evs[i], s);
        if (launch_decode_layer(d, ws->num_sms, s) == 0) {
            ws->launches += 1;
            ws->last_logit_cols = r->rows();
            for (int i = 4; evs && i <= 8; ++i) cudaEventRecord(evs[i], s);
            ws->last_rows = 0;  // no permuted accumulators to dump for this call
            ws->last_w = w;
            ws->last_stream = s;
            return cuda_rc(cudaPeekAtLastError());
        }
        cudaGetLastError();  // not launched: run the kernels one by one
    }
    // a small batch with a shared expert: its FFN starts before the router
    const bool side = (use_gemv(ws, w, rows) || use_w8_gemv(ws, w, rows)) && w->shared;
    if (side) {
        const int rc = start_shared_side(ws, w, rows, d_x, s);
        if (rc) {
            cudaStreamWaitEvent(s, ws->side_join, 0);
            return rc;
        }
    }
    const int rc = route_impl(ws, r, rows, d_x, nullptr, ws->ids, ws->routes, s);
    if (rc) {
        if (side) cudaStreamWaitEvent(s, ws->side_join, 0);
        return rc;
    }
    return run_pipeline(ws, w, rows, d_x, ws->ids, ws->routes, d_res, d_out, s, evs, res_ready,
                        router_gate(ws, r), side);
}

int moe_b200_forward_device(moe_b200_workspace* ws, const moe_b200_weights* w,
                            const moe_b200_router* r, int32_t rows, const float* d_input,
                            const float* d_residual, float* d_output, void* stream) {
    int rc = compatible(ws, w);
    if (rc) return rc;
    if (!r || r->H != ws->H || r->E != ws->E) return MOE_B200_ERR_INVALID;
    if (rows < 0) return MOE_B200_ERR_INVALID;
    if (rows > ws->max_rows) return MOE_B200_ERR_CAPACITY;
    if (rows == 0) return MOE_B200_OK;
    if (!d_input || !d_output || !aligned16(d_input) || !aligned16(d_residual) ||
        !aligned16(d_output))
        return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaEvent_t* evs = prof_slot(ws, 1 | (w->shared ? 2 : 0));
    if (evs) cudaEventRecord(evs[0], s);
    return layer_impl(ws, w, r, rows, d_input, d_residual, d_output, s, evs, nullptr);
}

struct moe_b200_graph {
    int device = 0;
    moe_b200_workspace* ws = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int64_t launches = 0;  // kernels per replay
};

moe_b200_graph* moe_b200_graph_create(moe_b200_workspace* ws, const moe_b200_weights* w,
                                      const moe_b200_router* r, int32_t rows,
                                      const float* d_input, const float* d_residual,
                                      float* d_output) {
    if (compatible(ws, w) || !r || r->H != ws->H || r->E != ws->E) return nullptr;
    if (rows <= 0 || rows > ws->max_rows || !d_input || !d_output || !aligned16(d_input) ||
        !aligned16(d_residual) || !aligned16(d_output))
        return nullptr;
    DeviceGuard guard(ws->device);
    cudaStream_t s = ws->own_stream;
    const bool prof = ws->profiling;
    ws->profiling = false;  // no event records inside the graph
    const int64_t l0 = ws->launches;
    int rc = MOE_B200_OK;
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        ws->profiling = prof;
        return nullptr;
    }
    rc = layer_impl(ws, w, r, rows, d_input, d_residual, d_output, s, nullptr, nullptr);
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    ws->profiling = prof;
    if (rc != MOE_B200_OK || e != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return nullptr;
    }
    cudaGraphExec_t x = nullptr;
    if (cudaGraphInstantiate(&x, g, 0) != cudaSuccess) {
        cudaGraphDestroy(g);
        return nullptr;
    }
    auto* out = new moe_b200_graph();
    out->device = ws->device;
    out->ws = ws;
    out->graph = g;
    out->exec = x;
    out->launches = ws->launches - l0;
    ws->launches = l0;  // replays count their kernels
    return out;
}

int moe_b200_graph_launch(moe_b200_graph* g, void* stream) {
    if (!g) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(g->device);
    g->ws->launches += g->launches;
    return cuda_rc(cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream)));
}

void moe_b200_graph_free(moe_b200_graph* g) {
    if (!g) return;
    DeviceGuard guard(g->device);
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
}

int64_t moe_b200_workspace_row_bytes(const moe_b200_workspace* ws) { return ws ? ws->Kh : 0; }

int moe_b200_ep_pack(moe_b200_workspace* ws, int32_t rows, const float* d_x, const int32_t* d_ids,
                     const float* d_routes, int32_t experts_per_rank, int32_t world,
                     int8_t* d_send_q, float* d_send_scale, int32_t* d_send_expert,
                     int32_t* d_send_counts, int32_t* d_pos, void* stream) {
    if (!ws || rows < 0 || experts_per_rank <= 0 || world <= 0 || world > 1024) return MOE_B200_ERR_INVALID;
    if (rows > ws->max_rows) return MOE_B200_ERR_CAPACITY;
    if (rows == 0) return MOE_B200_OK;
    if (!d_x || !d_ids || !d_routes || !d_send_q || !d_send_scale || !d_send_expert ||
        !d_send_counts || !d_pos || !aligned16(d_x) || !aligned16(d_send_q))
        return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int n = rows * ws->k;
    const int limit = experts_per_rank * world;
    ws->launches += 5;
    // group the assignments by destination rank (stable, assignment order)
    launch_route_count(d_ids, d_routes, n, world, ws->hist, ws->err, s, limit, experts_per_rank);
    launch_route_scatter(d_ids, d_routes, n, world, ws->hist, ws->offsets, ws->perm, d_pos,
                         nullptr, rows, s, limit, experts_per_rank);
    // quantise each token once and write its row into every kept slot
    launch_quant_gather(d_x, rows, ws->H, ws->Kh, kQuantMoe, ws->k, d_pos, nullptr, nullptr,
                        d_send_q, d_send_scale, nullptr, nullptr, ws->err, s);
    launch_ep_expert_ids(d_ids, d_pos, n, experts_per_rank, d_send_expert, s);
    // per-destination counts from the offsets
    launch_ep_counts(ws->offsets, world, d_send_counts, s);
    return cuda_rc(cudaPeekAtLastError());
}

// Expert side of the exchange on rows [n] (row stride ws->Kh): grouped by
// local expert, gate/up, requant, down into d_y in the received order. mask
// (may be null): rows with mask <= 0 are padding and skipped.
static int ep_expert_rows_impl(moe_b200_workspace* ws, const moe_b200_weights* w, int n,
                               const int8_t* d_q, const float* d_scale, const int32_t* d_expert,
                               const float* d_mask, float* d_y, cudaStream_t s) {
    const int E = ws->E, H = ws->H;
    ws->launches += 6;
    // stage events of the profiling ring: schedule+gather, gate/up, requant, down
    cudaEvent_t* evs = prof_slot(ws, 0);
    auto mark = [&](int i) {
        if (evs) cudaEventRecord(evs[i], s);
    };
    mark(0);
    mark(1);
    // rows -> permuted order by local expert (every kept row, one expert each)
    launch_route_count(d_expert, d_mask, n, E, ws->hist, ws->err, s);
    launch_route_scatter(d_expert, d_mask, n, E, ws->hist, ws->offsets, ws->perm, ws->pos,
                         nullptr, n, s);
    launch_ep_gather_rows(d_q, d_scale, ws->pos, n, ws->Kh, ws->a_perm, ws->s_perm, s);
    mark(2);
    mark(3);
    const int nt = choose_nt(n, E);
    const int nt_g = exact_nt(nt, w->gu.fmt);
    const int dfmt = down_fmt(w->dn.fmt, w->exact_down);
    const bool hd = dfmt == kFmtW4G32H;
    const int nt_d = exact_nt(nt, dfmt);
    {
        const int rc = run_gate_up(ws, w, n, nt_g, hd, s, mark);
        if (rc) return rc;
    }
    // down GEMM straight into the received order (permuted row p -> row perm[p])
    GemmArgs d = gemm_args(ws, w->dn, ws->s_m, ws->offsets, E, n, d_y, H);
    d.out_rows = ws->perm;
    if (launch_gemm(hd ? ws->map_qm_h[nt_index(nt_d)] : ws->map_qm[nt_index(nt_d)], d, dfmt,
                    kEpiStore, nt_d, ws->num_sms, s))
        return MOE_B200_ERR_UNSUPPORTED;
    mark(6);
    mark(7);
    mark(8);
    return cuda_rc(cudaPeekAtLastError());
}

int moe_b200_ep_expert_rows(moe_b200_workspace* ws, const moe_b200_weights* w, int32_t n,
                            const int8_t* d_q, const float* d_scale, const int32_t* d_expert,
                            float* d_y, void* stream) {
    int rc = compatible(ws, w);
    if (rc) return rc;
    if (w->shared) return MOE_B200_ERR_UNSUPPORTED;  // the owner computes the shared expert
    if (n < 0) return MOE_B200_ERR_INVALID;
    if (n > ws->n_max) return MOE_B200_ERR_CAPACITY;
    if (n == 0) return MOE_B200_OK;
    if (!d_q || !d_scale || !d_expert || !d_y || !aligned16(d_q) || !aligned16(d_y))
        return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    return ep_expert_rows_impl(ws, w, n, d_q, d_scale, d_expert, nullptr, d_y,
                               static_cast<cudaStream_t>(stream));
}

// ---- device-initiated exchange (peer memory) --------------------------------

struct moe_b200_ep_exchange {
    int device = 0, world = 0, rank = 0, cap = 0, H = 0;
    size_t row_bytes = 0, region_bytes = 0;
    uint8_t* region = nullptr;          // this rank's exchange region (exported)
    std::vector<uint8_t*> peers;        // every rank's region in this address space
    uint8_t** d_peers = nullptr;
    uint64_t* step = nullptr;
    int* done = nullptr;
    uint32_t* err = nullptr;
    float* mask = nullptr;              // [world * cap]
    float* y = nullptr;                 // [world * cap][H] expert rows of the received rows
    ExchangeArgs args{};
    bool connected = false;
    // stage events of profiled steps: begin, dispatched, rows arrived, expert
    // rows done, returned, returned rows arrived
    bool profiling = false;
    cudaEvent_t ev[6] = {};
};

moe_b200_ep_exchange* moe_b200_ep_exchange_create(int32_t device, int32_t world, int32_t rank,
                                                  int32_t cap, int64_t row_bytes, int32_t hidden) {
    if (world <= 0 || world > 64 || rank < 0 || rank >= world || cap <= 0 || hidden <= 0 ||
        hidden % 4 || row_bytes <= 0 || row_bytes % 16)
        return nullptr;
    if (check_device(device, nullptr)) return nullptr;
    DeviceGuard guard(device);
    auto* ex = new moe_b200_ep_exchange();
    ex->device = device;
    ex->world = world;
    ex->rank = rank;
    ex->cap = cap;
    ex->H = hidden;
    ex->row_bytes = (size_t)row_bytes;
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    ExchangeArgs& a = ex->args;
    const size_t wc = (size_t)world * cap;
    size_t off = 0;
    a.off_q = off;           off += al(wc * ex->row_bytes);
    a.off_scale = off;       off += al(wc * 4);
    a.off_expert = off;      off += al(wc * 4);
    a.off_cnt = off;         off += al((size_t)world * 4);
    a.off_base = off;        off += al((size_t)world * 4);
    a.off_y = off;           off += al((size_t)cap * hidden * 4);
    a.off_flag_rows = off;   off += al((size_t)world * 8);
    a.off_flag_y = off;      off += al((size_t)world * 8);
    ex->region_bytes = off;
    void* p = nullptr;
    bool ok = dev_alloc(&p, ex->region_bytes) == cudaSuccess;
    ex->region = static_cast<uint8_t*>(p);
    if (ok) ok = cudaMemset(ex->region, 0, ex->region_bytes) == cudaSuccess;
    auto get = [&](auto** dst, size_t bytes) {
        void* q = nullptr;
        if (!ok || dev_alloc(&q, bytes) != cudaSuccess || cudaMemset(q, 0, bytes) != cudaSuccess) {
            ok = false;
            return;
        }
        *dst = static_cast<std::remove_pointer_t<std::remove_reference_t<decltype(dst)>>>(q);
    };
    get(&ex->d_peers, sizeof(uint8_t*) * world);
    get(&ex->step, sizeof(uint64_t));
    get(&ex->done, sizeof(int));
    get(&ex->err, sizeof(uint32_t));
    get(&ex->mask, sizeof(float) * wc);
    get(&ex->y, sizeof(float) * wc * hidden);
    if (!ok) {
        moe_b200_ep_exchange_free(ex);
        return nullptr;
    }
    ex->peers.assign(world, nullptr);
    ex->peers[rank] = ex->region;
    a.peers = ex->d_peers;
    a.row_bytes = ex->row_bytes;
    a.world = world;
    a.rank = rank;
    a.cap = cap;
    a.H = hidden;
    a.blocks = 64;
    a.step = ex->step;
    a.done = ex->done;
    a.err = ex->err;
    return ex;
}

int moe_b200_ep_exchange_handle(const moe_b200_ep_exchange* ex, void* handle) {
    if (!ex || !handle) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ex->device);
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, ex->region);
    if (e != cudaSuccess) return cuda_rc(e);
    static_assert(sizeof(h) == MOE_B200_EP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    return MOE_B200_OK;
}

int moe_b200_ep_exchange_connect(moe_b200_ep_exchange* ex, const void* handles) {
    if (!ex || !handles || ex->connected) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ex->device);
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int r = 0; r < ex->world; ++r) {
        if (r == ex->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)r * MOE_B200_EP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_rc(e);
        ex->peers[r] = static_cast<uint8_t*>(p);
    }
    const cudaError_t e = cudaMemcpy(ex->d_peers, ex->peers.data(), sizeof(uint8_t*) * ex->world,
                                     cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_rc(e);
    ex->connected = true;
    return MOE_B200_OK;
}

int moe_b200_ep_exchange_step(moe_b200_ep_exchange* ex, moe_b200_workspace* ws,
                              const moe_b200_weights* w, const int8_t* d_send_q,
                              const float* d_send_scale, const int32_t* d_send_expert,
                              const int32_t* d_send_counts, void* stream) {
    if (!ex || !ex->connected) return MOE_B200_ERR_INVALID;
    int rc = compatible(ws, w);
    if (rc) return rc;
    if (w->shared) return MOE_B200_ERR_UNSUPPORTED;
    if (ws->device != ex->device || (size_t)ws->Kh != ex->row_bytes || ws->H != ex->H)
        return MOE_B200_ERR_INVALID;
    const long n = (long)ex->world * ex->cap;
    if (n > ws->n_max) return MOE_B200_ERR_CAPACITY;
    if (!d_send_q || !d_send_scale || !d_send_expert || !d_send_counts || !aligned16(d_send_q))
        return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ex->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const ExchangeArgs& a = ex->args;
    uint8_t* own = ex->region;
    auto mark = [&](int i) {
        if (ex->profiling) cudaEventRecord(ex->ev[i], s);
    };
    mark(0);
    launch_ep_begin(ex->step, s);
    launch_ep_dispatch(a, d_send_q, d_send_scale, d_send_expert, d_send_counts, s);
    mark(1);
    launch_ep_wait(a, 0, ex->mask, s);
    mark(2);
    rc = ep_expert_rows_impl(ws, w, (int)n, reinterpret_cast<const int8_t*>(own + a.off_q),
                             reinterpret_cast<const float*>(own + a.off_scale),
                             reinterpret_cast<const int32_t*>(own + a.off_expert), ex->mask, ex->y,
                             s);
    if (rc) return rc;
    mark(3);
    launch_ep_return(a, ex->y, s);
    mark(4);
    launch_ep_wait(a, 1, nullptr, s);
    mark(5);
    ws->launches += 5;
    return cuda_rc(cudaPeekAtLastError());
}

int moe_b200_ep_exchange_profile(moe_b200_ep_exchange* ex, int32_t enable) {
    if (!ex) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ex->device);
    if (enable && !ex->ev[0])
        for (auto& e : ex->ev)
            if (cudaEventCreate(&e) != cudaSuccess) return MOE_B200_ERR_CUDA;
    ex->profiling = enable != 0;
    return MOE_B200_OK;
}

int moe_b200_ep_exchange_profile_read(moe_b200_ep_exchange* ex, float* stage_us) {
    if (!ex || !stage_us || !ex->ev[0]) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ex->device);
    if (cudaEventSynchronize(ex->ev[5]) != cudaSuccess) return MOE_B200_ERR_CUDA;
    for (int i = 0; i < 5; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, ex->ev[i], ex->ev[i + 1]) != cudaSuccess)
            return MOE_B200_ERR_CUDA;
        stage_us[i] = 1000.0f * ms;
    }
    return MOE_B200_OK;
}

int moe_b200_ep_exchange_probe_timeout(moe_b200_ep_exchange* ex, void* stream) {
    if (!ex || !ex->connected || ex->world != 1) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ex->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    launch_ep_begin(ex->step, s);            // a step that no dispatch completes
    launch_ep_wait(ex->args, 0, nullptr, s);  // gives up after the wait limit
    return cuda_rc(cudaPeekAtLastError());
}

const float* moe_b200_ep_exchange_y_back(const moe_b200_ep_exchange* ex) {
    return ex ? reinterpret_cast<const float*>(ex->region + ex->args.off_y) : nullptr;
}

int moe_b200_ep_exchange_status(moe_b200_ep_exchange* ex) {
    if (!ex) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ex->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_rc(e);
    uint32_t bits = 0;
    e = cudaMemcpy(&bits, ex->err, sizeof(bits), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_rc(e);
    if (bits) cudaMemset(ex->err, 0, sizeof(uint32_t));
    return map_err_bits(bits);
}

void moe_b200_ep_exchange_free(moe_b200_ep_exchange* ex) {
    if (!ex) return;
    DeviceGuard guard(ex->device);
    cudaDeviceSynchronize();
    for (auto& e : ex->ev)
        if (e) cudaEventDestroy(e);
    for (int r = 0; r < (int)ex->peers.size(); ++r)
        if (r != ex->rank && ex->peers[r]) cudaIpcCloseMemHandle(ex->peers[r]);
    for (void* p : {(void*)ex->region, (void*)ex->d_peers, (void*)ex->step, (void*)ex->done,
                    (void*)ex->err, (void*)ex->mask, (void*)ex->y})
        if (p) cudaFree(p);
    delete ex;
}

int moe_b200_ep_combine(moe_b200_workspace* ws, int32_t rows, const float* d_y_back,
                        const int32_t* d_pos, const float* d_routes, const float* d_residual,
                        float* d_out, void* stream) {
    if (!ws || rows < 0) return MOE_B200_ERR_INVALID;
    if (rows > ws->max_rows) return MOE_B200_ERR_CAPACITY;
    if (rows == 0) return MOE_B200_OK;
    if (!d_y_back || !d_pos || !d_routes || !d_out || !aligned16(d_y_back) ||
        !aligned16(d_residual) || !aligned16(d_out))
        return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ws->launches += 1;
    launch_combine(d_y_back, d_pos, d_routes, nullptr, d_residual, rows, ws->H, ws->k, d_out, s);
    return cuda_rc(cudaPeekAtLastError());
}

int moe_b200_rms_norm(const float* d_x, const float* d_weight, int32_t rows, int32_t width,
                      float epsilon, int32_t zero_centered, float* d_out, void* stream) {
    // the reference's checks (src/ops/norm.rs:88-95): width > 0, finite eps > 0
    if (rows < 0 || width <= 0 || !(epsilon > 0.0f) || !std::isfinite(epsilon))
        return MOE_B200_ERR_INVALID;
    if (rows == 0) return MOE_B200_OK;
    if (!d_x || !d_weight || !d_out) return MOE_B200_ERR_INVALID;
    launch_rms_norm(d_x, d_weight, rows, width, epsilon, zero_centered != 0, d_out,
                    static_cast<cudaStream_t>(stream));
    return cuda_rc(cudaPeekAtLastError());
}

// The allocation id of page-locked host memory at p (0 for a null pointer),
// or false when p is not page-locked (copies from it cannot be captured).
static bool pinned_id(const void* p, unsigned long long* id) {
    *id = 0;
    if (!p) return true;
    static PFN_cuPointerGetAttribute_v4000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &f, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuPointerGetAttribute_v4000>(f);
    });
    if (!fn) return false;
    const CUdeviceptr_v2 a = (CUdeviceptr_v2)(uintptr_t)p;
    unsigned int type = 0;
    if (fn(&type, CU_POINTER_ATTRIBUTE_MEMORY_TYPE, a) != CUDA_SUCCESS ||
        type != CU_MEMORYTYPE_HOST)
        return false;
    return fn(id, CU_POINTER_ATTRIBUTE_BUFFER_ID, a) == CUDA_SUCCESS && *id != 0;
}

// The copies and the layer of a host-buffer call, on stream s; ev (the
// workspace's timing events, or null) brackets the stages.
static int enqueue_f32(moe_b200_workspace* ws, const moe_b200_weights* w, const moe_b200_router* r,
                       int rows, const float* input, const float* residual, float* output,
                       int32_t* ids, float* routes, cudaStream_t s, cudaEvent_t* ev) {
    const size_t xb = sizeof(float) * (size_t)rows * ws->H, nb = (size_t)rows * ws->k;
    if (ev) cudaEventRecord(ev[10], s);
    cudaMemcpyAsync(ws->x, input, xb, cudaMemcpyHostToDevice, s);
    // the residual is read only by the final combine: upload it beside the layer
    if (residual) {
        // after the input, which the router needs first: sharing the link from
        // the start would halve the input's rate and delay the whole layer
        cudaEventRecord(ws->x_ready, s);
        cudaStreamWaitEvent(ws->copy_stream, ws->x_ready, 0);
        cudaMemcpyAsync(ws->res, residual, xb, cudaMemcpyHostToDevice, ws->copy_stream);
        cudaEventRecord(ws->res_ready, ws->copy_stream);
    }
    if (ev) cudaEventRecord(ev[0], s);
    const int rc = layer_impl(ws, w, r, rows, ws->x, residual ? ws->res : nullptr, ws->out, s, ev,
                              residual ? ws->res_ready : nullptr);
    if (rc) {
        // the copy stream joins back (a capture ends only with every fork joined)
        if (residual) cudaStreamWaitEvent(s, ws->res_ready, 0);
        return rc;
    }
    cudaMemcpyAsync(output, ws->out, xb, cudaMemcpyDeviceToHost, s);
    if (ids) cudaMemcpyAsync(ids, ws->ids, sizeof(int32_t) * nb, cudaMemcpyDeviceToHost, s);
    if (routes) cudaMemcpyAsync(routes, ws->routes, sizeof(float) * nb, cudaMemcpyDeviceToHost, s);
    // the status word comes down with the outputs: one synchronisation per call
    cudaMemcpyAsync(ws->h_err, ws->err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
    if (ev) cudaEventRecord(ev[9], s);
    return MOE_B200_OK;
}

// A host-buffer call through the captured graph of its buffers (captured on
// the first call with these buffers; the key holds each buffer's address and
// page-locked allocation). MOE_B200_ERR_UNSUPPORTED when a buffer is not
// page-locked or the graph cannot be captured (the caller then runs the call
// eagerly).
static int forward_f32_graph(moe_b200_workspace* ws, const moe_b200_weights* w,
                             const moe_b200_router* r, int rows, const float* input,
                             const float* residual, float* output, int32_t* ids, float* routes) {
    cudaStream_t s = ws->own_stream;
    const void* host[5] = {input, residual, output, ids, routes};
    uint64_t key[12] = {w->serial, r->serial};
    for (int i = 0; i < 5; ++i) {
        unsigned long long id = 0;
        if (!pinned_id(host[i], &id)) return MOE_B200_ERR_UNSUPPORTED;
        key[2 + 2 * i] = (uint64_t)(uintptr_t)host[i];
        key[3 + 2 * i] = id;
    }
    auto& hg = ws->hg;
    bool hit = (hg.exec || hg.failed) && hg.rows == rows;
    for (int i = 0; i < 12 && hit; ++i) hit = hg.key[i] == key[i];
    if (hit && hg.failed) return MOE_B200_ERR_UNSUPPORTED;
    if (!hit) {
        if (hg.exec) cudaGraphExecDestroy(hg.exec);
        if (hg.graph) cudaGraphDestroy(hg.graph);
        hg = moe_b200_workspace::HostGraph{};
        const int64_t l0 = ws->launches;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            cudaGetLastError();
            return MOE_B200_ERR_UNSUPPORTED;
        }
        const int rc = enqueue_f32(ws, w, r, rows, input, residual, output, ids, routes, s, nullptr);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(s, &g);
        const int64_t launched = ws->launches - l0;
        ws->launches = l0;
        cudaGraphExec_t x = nullptr;
        for (int i = 0; i < 12; ++i) hg.key[i] = key[i];
        hg.rows = rows;
        if (rc || e != cudaSuccess || !g || cudaGraphInstantiate(&x, g, 0) != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            hg.failed = !rc;
            return rc ? rc : MOE_B200_ERR_UNSUPPORTED;
        }
        hg.graph = g;
        hg.exec = x;
        hg.launches = launched;
    }
    ws->launches += hg.launches;
    cudaError_t e = cudaGraphLaunch(hg.exec, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_rc(e);
    ws->last_stream = s;
    return handle_status(ws, *ws->h_err, s);
}

int moe_b200_forward_f32(moe_b200_workspace* ws, const moe_b200_weights* w,
                         const moe_b200_router* r, int32_t rows, const float* input,
                         const float* residual, float* output, int32_t* ids, float* routes,
                         moe_b200_timings* timings) {
    int rc = compatible(ws, w);
    if (rc) return rc;
    if (!r || r->H != ws->H || r->E != ws->E) return MOE_B200_ERR_INVALID;
    if (rows < 0) return MOE_B200_ERR_INVALID;
    if (rows > ws->max_rows) return MOE_B200_ERR_CAPACITY;
    if (rows == 0) return MOE_B200_OK;
    if (!input || !output) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    cudaStream_t s = ws->own_stream;
    // page-locked buffers, no timings: the captured copies + layer of these
    // buffers (one launch, no per-kernel launch gaps)
    if (!timings && !ws->profiling) {
        const int grc = forward_f32_graph(ws, w, r, rows, input, residual, output, ids, routes);
        if (grc != MOE_B200_ERR_UNSUPPORTED) return grc;
    }
    rc = enqueue_f32(ws, w, r, rows, input, residual, output, ids, routes, s,
                     timings ? ws->ev : nullptr);
    if (rc) return rc;
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_rc(e);
    rc = handle_status(ws, *ws->h_err, s);
    if (timings) {
        fill_timings(ws, timings, rows, true, w->shared != 0);
        timings->sync_us = 1000.0 * ev_ms(ws->ev[8], ws->ev[9]);
        timings->total_us = 1000.0 * ev_ms(ws->ev[10], ws->ev[9]);
    }
    return rc;
}

int moe_b200_workspace_status(moe_b200_workspace* ws) {
    if (!ws) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    // the last launching stream (a null handle is the legacy default stream,
    // which the non-blocking own stream does not order against), then our own
    cudaError_t e = cudaStreamSynchronize(ws->last_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ws->own_stream);
    if (e != cudaSuccess) return cuda_rc(e);
    return read_status(ws, ws->own_stream);
}

int moe_b200_workspace_buffer(moe_b200_workspace* ws, const char* name, void** d_ptr,
                              uint64_t* bytes) {
    if (!ws || !name || !d_ptr) return MOE_B200_ERR_INVALID;
    const long T = ws->max_rows, n = ws->n_max;
    struct Entry {
        const char* name;
        void* p;
        uint64_t b;
    } table[] = {
        {"q_x", ws->q_x, (uint64_t)T * ws->Kh},
        {"s_x", ws->s_x, sizeof(float) * (uint64_t)T},
        {"perm", ws->perm, sizeof(int32_t) * (uint64_t)n},
        {"pos", ws->pos, sizeof(int32_t) * (uint64_t)n},
        {"offsets", ws->offsets, sizeof(int32_t) * (uint64_t)(ws->E + 1)},
        {"a_perm", ws->a_perm, (uint64_t)n * ws->Kh},
        {"s_perm", ws->s_perm, sizeof(float) * (uint64_t)n},
        {"gate_up", ws->gate_up, sizeof(float) * (uint64_t)n * 2 * ws->I},
        {"q_m", ws->q_m, (uint64_t)n * ws->Ki},
        {"s_m", ws->s_m, sizeof(float) * (uint64_t)n},
        {"y", ws->y, sizeof(float) * (uint64_t)n * ws->H},
        {"shared_y", ws->s_y, ws->s_y ? sizeof(float) * (uint64_t)T * ws->H : 0},
        {"logits", ws->logits,
         sizeof(float) * (uint64_t)T * (ws->last_logit_cols ? ws->last_logit_cols : ws->E)},
        {"ids", ws->ids, sizeof(int32_t) * (uint64_t)n},
        {"routes", ws->routes, sizeof(float) * (uint64_t)n},
    };
    for (const Entry& e : table)
        if (strcmp(e.name, name) == 0) {
            if (!e.p) return MOE_B200_ERR_INVALID;
            *d_ptr = e.p;
            if (bytes) *bytes = e.b;
            return MOE_B200_OK;
        }
    return MOE_B200_ERR_INVALID;
}

int moe_b200_debug_accumulators(moe_b200_workspace* ws, const moe_b200_weights* w, int32_t which,
                                int32_t* d_acc, uint64_t capacity_elems, void* stream) {
    int rc = compatible(ws, w);
    if (rc) return rc;
    if (!d_acc || (which != 0 && which != 1) || ws->last_w != w || ws->last_rows <= 0)
        return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const PackedMat& m = which == 0 ? w->gu : w->dn;
    const long n = (long)ws->last_rows * ws->k;
    const int G = m.fmt == kFmtW4G32 ? m.kblocks * 4 : 1;
    const int ld = which == 0 ? 2 * w->I : w->H;
    if ((uint64_t)n * G * ld > capacity_elems) return MOE_B200_ERR_CAPACITY;
    cudaMemsetAsync(d_acc, 0, sizeof(int32_t) * (size_t)n * G * ld, s);
    const int nt = exact_nt(which == 0 ? ws->last_nt_gu : ws->last_nt_dn, m.fmt);
    GemmArgs a = which == 0 ? gemm_args(ws, m, ws->s_perm, ws->offsets, ws->E, n, nullptr, 0)
                            : gemm_args(ws, m, ws->s_m, ws->offsets, ws->E, n, nullptr, 0);
    a.acc_out = d_acc;
    a.acc_ld = ld;
    a.n_valid = which == 0 ? w->I : w->H;
    const CUtensorMap& map = which == 0 ? ws->map_a[nt_index(nt)] : ws->map_qm[nt_index(nt)];
    if (launch_gemm(map, a, m.fmt, kEpiAcc, nt, ws->num_sms, s)) return MOE_B200_ERR_UNSUPPORTED;
    return cuda_rc(cudaPeekAtLastError());
}

int moe_b200_workspace_profile(moe_b200_workspace* ws, int32_t enable) {
    if (!ws) return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    if (enable && ws->prof_ev.empty()) {
        const size_t n = (size_t)moe_b200_workspace::kProfSlots * moe_b200_workspace::kProfEvents;
        ws->prof_ev.resize(n, nullptr);
        for (size_t i = 0; i < n; ++i)
            if (cudaEventCreate(&ws->prof_ev[i]) != cudaSuccess) return MOE_B200_ERR_CUDA;
        ws->prof_flags.assign(moe_b200_workspace::kProfSlots, 0);
    }
    ws->profiling = enable != 0;
    ws->prof_calls = 0;
    return MOE_B200_OK;
}

int moe_b200_workspace_profile_read(moe_b200_workspace* ws, int32_t call, moe_b200_timings* t) {
    if (!ws || !t || ws->prof_ev.empty() || call < 0 || call >= ws->prof_calls ||
        call < ws->prof_calls - moe_b200_workspace::kProfSlots)
        return MOE_B200_ERR_INVALID;
    DeviceGuard guard(ws->device);
    const int slot = call % moe_b200_workspace::kProfSlots;
    const cudaEvent_t* ev = &ws->prof_ev[(size_t)slot * moe_b200_workspace::kProfEvents];
    cudaError_t e = cudaEventSynchronize(ev[8]);
    if (e != cudaSuccess) return cuda_rc(e);
    const int fl = ws->prof_flags[slot];
    fill_timings_from(ev, ws, t, ws->last_rows, (fl & 1) != 0, (fl & 2) != 0);
    return MOE_B200_OK;
}

int64_t moe_b200_workspace_launches(const moe_b200_workspace* ws) { return ws ? ws->launches : 0; }

const char* moe_b200_strerror(int code) {
    switch (code) {
        case MOE_B200_OK: return "success";
        case MOE_B200_ERR_INVALID: return "invalid argument or shape";
        case MOE_B200_ERR_UNSUPPORTED: return "shape or format not supported by this build";
        case MOE_B200_ERR_NOMEM: return "device memory allocation failed";
        case MOE_B200_ERR_CUDA: return "CUDA runtime error";
        case MOE_B200_ERR_CAPACITY: return "rows exceed the workspace max_rows";
        case MOE_B200_ERR_DEVICE_TIMEOUT: return "a bounded device wait timed out";
        case MOE_B200_ERR_BAD_EXPERT: return "expert id out of range";
        case MOE_B200_ERR_NONFINITE: return "non-finite router logit or activation";
        case MOE_B200_ERR_BAD_ROUTE: return "negative or NaN routing weight";
        case MOE_B200_ERR_NO_DEVICE: return "no sm_100 CUDA device available";
        case MOE_B200_ERR_NOALLOC_LIMIT:
            return "rows * experts exceed the fixed scratch of the no-allocation router";
        default: return "unknown error";
    }
}

const char* moe_b200_version(void) { return "moe_b200 0.1.0 sm_100a"; }

}  // extern "C"
