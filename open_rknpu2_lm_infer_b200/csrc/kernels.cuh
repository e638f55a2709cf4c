// Kernel entry points and argument blocks shared by the C ABI (api.cu) and
// the kernel translation units.
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace moe {

// Weight formats (values 0..2 match MOE_B200_W* in include/moe_b200.h).
// kFmtW4G32 runs on the int8 tensor cores with one exact int32 sum per group
// (the accumulator dump); kFmtW4G32H is the same packed bank on the fp16
// tensor cores: the unpack warps write w * s_group (one fp16 rounding) and
// the MMA accumulates all of K in fp32, one accumulator per tile.
enum { kFmtW4PC = 0, kFmtW4G32 = 1, kFmtW8PC = 2, kFmtW4G32H = 3 };
// GEMM epilogues. GateUp: a gate/up tile (64 gate + 64 up channels) stores its
// dequantised values as gate | up halves of a [rows][2n] row, the layout the
// SwiGLU of the requantisation kernel reads. Store: [rows][n]. Acc: int32 dump.
enum { kEpiGateUp = 0, kEpiStore = 1, kEpiAcc = 2 };
// Activation quantisation rules.
enum { kQuantMoe = 0, kQuantDense = 1 };

// Routing rules: softmax over the top-k logits (Qwen), and grouped sigmoid
// top-k with a selection bias (Ling).
enum { kRouteSoftmax = 0, kRouteGroupedSigmoid = 1 };
// Router dot orders (values match MOE_B200_ROUTER_*).
enum { kOrderNeon16 = 0, kOrderSequential = 1, kOrderTf32 = 2 };

struct RouterArgs {
    const float* x;       // [T][H]
    const float* w;       // [Ew][H]: E expert rows, then the shared-gate row if any
    const float* bias;    // [E] added to the logits, or null
    int T, H, E, k, order;
    int Ew;               // weight rows = logits row stride (0 means E)
    float min_weight;
    float* logits;        // [T][Ew] scratch / output
    int* counters;        // [ceil(T)] zeroed tile counters
    int32_t* ids;         // [T][k]
    float* weights;       // [T][k]
    uint32_t* err;
    // grouped sigmoid rule
    int rule;             // kRoute*
    const float* sel_bias;  // [E] selection bias
    int groups, top_groups;
    float scale;          // routing scale
};
constexpr int kGroupedMaxExperts = 256;  // grouped sigmoid: E <= 8 per lane of a warp

struct GemmArgs {
    const float* act_scale;   // per permuted row
    const int32_t* offsets;   // [E+1] row ranges of the permuted activations
    int num_experts;
    int max_rows;             // upper bound of offsets[E] (grid sizing)
    const uint8_t* w;         // tile-major packed weights
    size_t w_expert_stride;   // bytes
    size_t w_tile_stride;     // bytes per 128-row tile (all k-blocks)
    size_t w_stage_stride;    // bytes per load stage within a tile
    const void* wscale;       // scales, tile-major
    size_t ws_expert_stride;  // bytes
    size_t ws_tile_stride;    // bytes
    int kblocks;              // K / 128
    int row_tiles;            // weight row tiles of 128
    float* out;               // GateUp: gate | up [rows][ldo = 2n]; Store: y [rows][ldo]
    const int32_t* out_rows;  // Store: output row of each permuted row (null: the same)
    int ldo;
    int n_valid;              // valid output channels (I or H)
    int32_t* acc_out;         // accumulator dump
    int acc_ld;               // row length of the dump (n or 2I)
    int swiglu_layout;        // dump channel mapping of the gate/up tiles
    uint32_t* err;
};


// -1 (nothing launched) when the geometry does not fit: see router_fits.
int launch_router(const RouterArgs& a, cudaStream_t s);
// Whether launch_router can run `rows` tokens of width `hidden` in dot order
// `order`: the NEON16 / TF32 orders at fewer than 16 tokens stage 8 router
// rows and the token in shared memory (<= 200 KiB).
bool router_fits(int rows, int hidden, int order);
int launch_gemm(const CUtensorMap& map, const GemmArgs& a, int fmt, int epi, int nt,
                int num_sms, cudaStream_t s);

// dispatch.cu
// Grouping of assignments by key = id / div (ids in [0, id_limit), default E;
// routes == nullptr keeps every assignment): stable ranks, offsets [E+1],
// perm (slot -> assignment), pos (assignment -> slot or -1).
void launch_route_count(const int32_t* ids, const float* routes, int n, int E, int32_t* hist,
                        uint32_t* err, cudaStream_t s, int id_limit = 0, int div = 1);
void launch_route_scatter(const int32_t* ids, const float* routes, int n, int E,
                          const int32_t* hist, int32_t* offsets, int32_t* perm, int32_t* pos,
                          int32_t* shared_offsets, int T, cudaStream_t s, int id_limit = 0,
                          int div = 1);
// expert parallelism helpers
void launch_ep_expert_ids(const int32_t* ids, const int32_t* pos, int n, int per_rank,
                          int32_t* send_expert, cudaStream_t s);
void launch_ep_counts(const int32_t* offsets, int world, int32_t* counts, cudaStream_t s);
void launch_ep_gather_rows(const int8_t* q, const float* scale, const int32_t* pos, int n, int ld,
                           int8_t* q_perm, float* s_perm, cudaStream_t s);
// h_rows / h_perm / qh (may be null): the same codes as fp16, for kFmtW4G32H.
void launch_quant_gather(const float* x, int T, int H, int ld_q, int rule, int k,
                         const int32_t* pos, int8_t* q_rows, float* s_rows, int8_t* q_perm,
                         float* s_perm, __half* h_rows, __half* h_perm, uint32_t* err,
                         cudaStream_t s);
void launch_requant(const float* gate_up, const int32_t* count, int max_rows, int I, int ld_q,
                    int rule, int8_t* q, __half* qh, float* sc, cudaStream_t s);
// gate (may be null): the shared-gate logit of token t at gate[t * gate_ld];
// the shared row then enters as sigmoid(gate) * shared.
// offsets[0] = 0, offsets[1] = rows: the one-expert grouping of the shared
// expert when no routed grouping ran.
void launch_set_range(int32_t* offsets, int rows, cudaStream_t s);
void launch_combine(const float* y, const int32_t* pos, const float* routes, const float* shared,
                    const float* residual, int T, int H, int k, float* out, cudaStream_t s,
                    const float* gate = nullptr, int gate_ld = 0);

// gemv_w8.cu: the small-batch FFN of a per-channel int8 bank (one expert: the
// shared expert), split-K GEMVs. Gate/up: grid (row tiles, load stages),
// out = the SwiGLU middle [T][n], then the middle's codes q_out [T][ld_q] and
// scales q_scale under `rule`; down: out = the expert rows [T][n].
struct W8GemvArgs {
    const uint8_t* w;          // packed bank (one expert)
    size_t w_tile_stride, w_stage_stride;
    const void* wscale;        // per-channel f32 scales, tile-major
    size_t ws_tile_stride;     // bytes
    const int8_t* q;           // [T][ld] activation codes
    int ld;
    const float* sx;           // [T] activation scales
    int T, n;
    int32_t* acc;              // [T][row tiles * 128] zero, re-zeroed
    int* counters;             // [row tiles + 1] zero, re-zeroed
    uint32_t* row_max;         // [T] zero, re-zeroed (gate/up)
    float* out;
    int8_t* q_out;
    float* q_scale;
    int ld_q, rule;
    uint32_t* err;
};
int launch_shared_w8(const W8GemvArgs& a, bool gateup, int row_tiles, int kstages, cudaStream_t s);

// gemv_w8.cu: the routed experts of a per-channel int8 bank at one to four
// tokens, the same split-K GEMVs per kept assignment: gate/up (the token's
// MoE A8 codes, SwiGLU, the middle's codes) into q_m / s_m, then down with
// the last-arrival combine of a (token, 128-channel tile): the kept ranks in
// rank order, the shared row (sigmoid-gated if gate), the residual.
struct W8RoutedArgs {
    const int32_t* ids;        // [T][k]
    const float* routes;       // [T][k]
    int T, k, E, H, I;
    int gu_stages, dn_stages;  // 256-k load stages of the two banks
    const float* x;            // [T][H]
    const uint8_t* gu_w;       // packed gate|up bank
    size_t gu_expert_stride, gu_tile_stride, gu_stage_stride;
    const float* gu_s;         // per-channel scales
    size_t gu_s_expert_stride, gu_s_tile_stride;
    const uint8_t* dn_w;
    size_t dn_expert_stride, dn_tile_stride, dn_stage_stride;
    const float* dn_s;
    size_t dn_s_expert_stride, dn_s_tile_stride;
    int32_t* acc;              // [T*k][max(2I, H) padded] zero, re-zeroed
    int* counters;             // [T*k*(gu tiles + 1 + dn tiles) + T*dn tiles] zero, re-zeroed
    uint32_t* row_max;         // [T*k] zero, re-zeroed
    float* middle;             // [T*k][I]
    int8_t* q_m;               // [T*k][ld_qm]
    float* s_m;                // [T*k]
    int ld_qm;
    float* y;                  // [T*k][H]
    const float* shared;       // [T][H] or null
    const float* gate;         // shared-gate logits or null
    int gate_ld;
    const float* residual;     // [T][H] or null
    float* out;                // [T][H]
    uint32_t* err;
};
int launch_routed_w8(const W8RoutedArgs& a, int part, cudaStream_t s);

// gemv.cu: the small-batch path of group-32 int4 banks (a shared expert, if
// any, runs beside it and enters the combine of the down kernel).
struct GemvArgs {
    const int32_t* ids;       // [T][k]
    const float* routes;      // [T][k]
    int T, k, E, H, I;
    const float* x;           // [T][H] activations (quantised in the gate/up kernel)
    const uint8_t* gu_w;      // packed gate|up bank
    size_t gu_expert_stride, gu_tile_stride, gu_stage_stride;
    int gu_stages;            // 256-k stages of the gate/up K (= H padded)
    const uint8_t* dn_w;      // packed down bank
    size_t dn_expert_stride, dn_tile_stride, dn_stage_stride;
    int dn_stages;
    float* middle;            // [T*k][I]
    int8_t* q_m;              // [T*k][ld_qm]
    float* s_m;               // [T*k]
    int ld_qm;
    float* y;                 // [T*k][H]
    const float* residual;    // [T][H] or null
    float* out;               // [T][H]
    int* counters;            // [T*k] gate/up, then [T][H/128] down (zeroed)
    int dn_counter_base;
    const float* shared;      // [T][H] shared-expert rows added after the ranks, or null
    const float* gate;        // shared-gate logits gate[t * gate_ld] (sigmoid scale), or null
    int gate_ld;
    uint32_t* err;
};
// part 0: gate/up (+ SwiGLU + requant), part 1: down (+ combine + residual).
// -1 when the stage set does not fit shared memory (kGemvMaxSmem).
constexpr size_t kGemvMaxSmem = 220 * 1024;
int launch_gemv(const GemvArgs& a, int part, cudaStream_t s);
size_t gemv_smem_bytes(int stages);

// gemv.cu: the whole small-batch layer in one cooperative launch: router
// logits, routing, gate/up + SwiGLU, requantisation, down, combine + residual,
// with one grid-wide barrier after the logits and per-assignment ready counts
// between gate/up and down (bounded waits). -1 when the geometry does not fit
// (the caller then runs the router and the two GEMV kernels).
struct DecodeArgs {
    RouterArgs r;              // logits scratch; ids / weights outputs
    GemvArgs g;                // ids / routes = r.ids / r.weights
    uint32_t* mmax;            // [T*k] bits of each middle row's max |value| (zeroed by the kernel)
    uint32_t* ready;           // [T*k] gate/up items done per assignment (zeroed by the kernel)
    unsigned long long* bar;   // grid barrier counters [8 x 16], each at a multiple of its CTAs at rest
};
int launch_decode_layer(const DecodeArgs& d, int num_sms, cudaStream_t s);

// exchange.cu: device-initiated expert-parallel exchange (peer memory).
struct ExchangeArgs {
    uint8_t* const* peers;    // [world] exchange regions, this rank's at [rank]
    size_t off_q, off_scale, off_expert, off_cnt, off_base, off_y, off_flag_rows, off_flag_y;
    size_t row_bytes;
    int world, rank, cap, H, blocks;
    const uint64_t* step;     // this step's number (local)
    int* done;                // last-CTA counter (local, zeroed)
    uint32_t* err;            // status word (local)
};
void launch_ep_begin(uint64_t* step, cudaStream_t s);
void launch_ep_dispatch(const ExchangeArgs& a, const int8_t* send_q, const float* send_scale,
                        const int32_t* send_expert, const int32_t* counts, cudaStream_t s);
// which = 0: rows (fills mask [world * cap] with 1 / 0), 1: returned y rows.
void launch_ep_wait(const ExchangeArgs& a, int which, float* mask, cudaStream_t s);
void launch_ep_return(const ExchangeArgs& a, const float* y, cudaStream_t s);

// Exchanges two device byte ranges (16-byte aligned, bytes % 16 == 0).
void launch_swap_bytes(void* a, void* b, size_t bytes, cudaStream_t s);
// RMSNorm rows (norm.cu); x and out may alias.
void launch_rms_norm(const float* x, const float* w, int rows, int width, float eps,
                     int zero_centered, float* out, cudaStream_t s);

constexpr int kRouteChunk = 512;  // assignments per route_count / route_scatter CTA

// K-blocks (128 bytes of K each) per GEMM load stage: one bulk copy brings the
// stage's weights (and group scales), one 3-D tensor copy its activations.
// A copy request costs a fixed ~0.2 us per SM, so stages move >= 16 KB.
constexpr int kKPS = 2;
constexpr int kKAlign = 128 * kKPS;  // K padding of weights and activation rows

}  // namespace moe
