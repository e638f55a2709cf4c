/*
 * moe_b200 — B200 (sm_100a) MoE feed-forward operator, C ABI.
 *
 * Drop-in replacement for the grouped-MoE operator surface that the
 * happyme531/open_rknpu2_lm_infer Rust crate binds through bindgen
 * (build.rs:137-145 over the absent native/rk_npu_matmul include/rk_npu_moe_w8.h;
 * call sites in src/npu/moe.rs and src/npu.rs). Each declaration names the
 * reference entry point it replaces. Plain pointers and sizes only; every
 * function returns 0 on success or a negative MOE_B200_ERR_* code, and
 * creators return NULL on failure (as Handle::new expects, src/npu.rs:176-180).
 *
 * Weight layout at the boundary is the reference's QuantMatrix
 * (src/npu.rs:135-157): codes int8 [k][n] (row k holds the n output channels),
 * f32 per-output-channel scales [n]. gate_up has n = 2*intermediate with the
 * gate columns first (src/model/checkpoint.rs:573-605); down has k =
 * intermediate, n = hidden. The group-32 fp16 scale format is an extension
 * (the reference loader rejects group scales, src/model/checkpoint.rs:251-263).
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- error codes (rk_npu_strerror convention, src/npu.rs:187-193) ------- */
#define MOE_B200_OK 0
#define MOE_B200_ERR_INVALID (-1)       /* bad argument / shape */
#define MOE_B200_ERR_UNSUPPORTED (-2)   /* shape or format outside this build */
#define MOE_B200_ERR_NOMEM (-3)         /* device or host allocation failed */
#define MOE_B200_ERR_CUDA (-4)          /* CUDA runtime error */
#define MOE_B200_ERR_CAPACITY (-5)      /* rows above the workspace max_rows */
#define MOE_B200_ERR_DEVICE_TIMEOUT (-6) /* a bounded device wait gave up */
#define MOE_B200_ERR_BAD_EXPERT (-7)    /* expert id outside [0, experts) */
#define MOE_B200_ERR_NONFINITE (-8)     /* non-finite router logit / activation */
#define MOE_B200_ERR_BAD_ROUTE (-9)     /* negative or NaN routing weight */
#define MOE_B200_ERR_NO_DEVICE (-10)    /* no sm_100 device / library built without it */
#define MOE_B200_ERR_NOALLOC_LIMIT (-11) /* request larger than the fixed no-allocation scratch */

/* Routed-expert weight formats. */
#define MOE_B200_W4_PER_CHANNEL 0 /* reference native format: int4 codes, f32 scale per n */
/* int4 codes, fp16 scale per (32 k, n) group (an extension: the reference
 * loader rejects group scales, src/model/checkpoint.rs:251-263). Both GEMMs
 * keep one exact int32 sum per group and fold them in f32 in group order:
 * f = fma((float)acc_g, s_g, f), then * s_x. */
#define MOE_B200_W4_G32_FP16 1
#define MOE_B200_W8_PER_CHANNEL 2 /* int8 codes, f32 scale per n */
/* The same as MOE_B200_W4_G32_FP16 (kept for callers of an earlier version). */
#define MOE_B200_W4_G32_FP16_EXACT 3
/* The group-32 bank with the down GEMM on the fp16 tensor cores instead: w * s
 * rounded once to fp16, fp32 accumulation over all of K. No int32 down
 * accumulators; outputs stay within 1e-2 rel / 1e-3 abs of the exact format.
 * The gate/up GEMM stays exact (its output is requantised). Opt-in. */
#define MOE_B200_W4_G32_FP16_ROUNDED_DOWN 4

/* Router accumulation order (src/model/cpu.rs:96-153, dense_dot). */
#define MOE_B200_ROUTER_NEON16 0     /* aarch64 F32 branch: 4x4-lane FMA + fixed tree */
#define MOE_B200_ROUTER_SEQUENTIAL 1 /* x86 scalar loop: separately rounded mul + add */
#define MOE_B200_ROUTER_TF32 2       /* Ling's TF32 linear (src/npu/tf32.rs): operands
                                        narrowed to TF32, f32 sums (within 5e-5 of the
                                        f64 sum, the reference's own bound) */

/* Routing rules. */
#define MOE_B200_ROUTE_SOFTMAX 0          /* routes(), src/model/qwen35/moe.rs:51-67 */
#define MOE_B200_ROUTE_GROUPED_SIGMOID 1  /* Ling, src/model/ling3tiny/moe.rs:146-223 */

/* Shared expert arithmetic. */
#define MOE_B200_SHARED_JOINT 0 /* MoE input quantisation, nearest-even (joint bank) */
#define MOE_B200_SHARED_DENSE 1 /* separate dense W8A8 FFN, round-away quantisation */

typedef struct moe_b200_weights moe_b200_weights;
typedef struct moe_b200_workspace moe_b200_workspace;
typedef struct moe_b200_router moe_b200_router;

/* Replaces rk_npu_moe_w8_weight_config (fields used at src/npu/moe.rs:245-250). */
typedef struct {
    int32_t hidden;
    int32_t intermediate;
    int32_t routed_experts;
    int32_t shared_expert;        /* 0 or 1 */
    int32_t shared_intermediate;  /* extension; 0 = same as intermediate */
} moe_b200_weight_config;

/* Replaces rk_npu_moe_w8_config (src/npu/moe.rs:179-192). npu_cores and
 * cpu_threads have no meaning here and are kept only for source parity. */
typedef struct {
    moe_b200_weight_config weights;
    int32_t top;
    int32_t max_rows;      /* the reference's `chunk` (Moe::max_rows) */
    int32_t device;        /* CUDA device ordinal */
    int32_t npu_cores;     /* ignored */
    int32_t cpu_threads;   /* ignored */
} moe_b200_config;

/* Replaces rk_npu_moe_w8_expert (src/npu/moe.rs:121-126). The *_group_scales
 * pointers are read only for the group-32 formats: IEEE fp16 bits laid out
 * [k/32][n]. */
typedef struct {
    const int8_t *gate_up;
    const float *gate_up_scales;
    const int8_t *down;
    const float *down_scales;
    const uint16_t *gate_up_group_scales;
    const uint16_t *down_group_scales;
} moe_b200_expert;

/* Extension: weight formats of one bank. */
typedef struct {
    int32_t routed_format;  /* MOE_B200_W4_* / MOE_B200_W8_* */
    int32_t shared_format;  /* MOE_B200_W8_PER_CHANNEL or MOE_B200_W4_PER_CHANNEL */
    int32_t shared_mode;    /* MOE_B200_SHARED_* */
} moe_b200_format;

/* Replaces rk_npu_moe_w8_timings (fields read at src/npu/moe.rs:342-351).
 * Filled from CUDA events: input_us = activation quantisation, schedule_us =
 * route histogram + permutation, gather_us = row gather, gate_us = gate/up
 * GEMM, middle_cpu_us = SwiGLU + middle requantisation, down_us = down GEMM,
 * combine_us = weighted combine (+ shared + residual), build_us = shared
 * expert, total_us = whole call. Counters are work items of the launch. */
typedef struct {
    double input_us, schedule_us, build_us, sync_us, gather_us, gate_us;
    double middle_npu_us, middle_cpu_us, down_us, combine_us, lut_load_us, total_us;
    int64_t gather_tasks, middle_tasks, gemm_tasks;
    double router_us; /* extension: router logits + top-k (forward only) */
} moe_b200_timings;

/* ---- configuration / objects ------------------------------------------- */

/* Replaces rk_npu_moe_w8_config_init(cfg, h, f, e, shared, top, chunk). */
void moe_b200_config_init(moe_b200_config *cfg, int32_t hidden, int32_t intermediate,
                          int32_t experts, int32_t shared, int32_t top, int32_t max_rows);

/* Replaces rk_npu_moe_quant_weights_create / _full_k / rk_npu_moe_w4_weights_create
 * (src/npu/moe.rs:131-139). experts[routed_experts] (+ experts[routed_experts]
 * = the shared expert when shared_expert = 1, as at src/npu/moe.rs:128-130).
 * Host arrays are copied and packed; the caller may free them afterwards. */
moe_b200_weights *moe_b200_weights_create(const moe_b200_config *cfg,
                                          const moe_b200_expert *experts,
                                          const moe_b200_format *format);
/* Replaces rk_npu_moe_w8_weights_free. */
void moe_b200_weights_free(moe_b200_weights *w);
/* Replaces rk_npu_moe_w8_weights_device_bytes. */
uint64_t moe_b200_weights_device_bytes(const moe_b200_weights *w);

/* ---- expert slot bank (replaces rk_npu_moe_quant_slots_create,
 * _expert_blob_bytes, _export_expert, _import_expert and _swap_slots, used by
 * Moe::import_bank / promote / export / import at src/npu/moe.rs:243-320).
 * A blob is one routed expert's packed device image: a 64-byte header (magic
 * "MB2XBLOB", MOE_B200_BLOB_VERSION, format, hidden, intermediate, four
 * region sizes) followed by the bank's own gate|up and down regions, so
 * export and import are plain copies. Blobs are specific to this library's
 * packing and to the bank's format and geometry; a mismatch is
 * MOE_B200_ERR_INVALID. ------------------------------------------------- */
#define MOE_B200_BLOB_VERSION 1
uint32_t moe_b200_blob_version(void);
/* An empty routed bank of cfg->weights.routed_experts slots in routed_format
 * (MOE_B200_W4_*, MOE_B200_W8_*); zero weights; no shared expert. */
moe_b200_weights *moe_b200_slots_create(const moe_b200_config *cfg, int32_t routed_format);
uint64_t moe_b200_expert_blob_bytes(const moe_b200_weights *w);
/* Synchronous device -> host copy of expert `expert`; bytes must equal the blob size. */
int moe_b200_export_expert(const moe_b200_weights *w, int32_t expert, void *data, uint64_t bytes);
/* Synchronous host -> device copy into slot `slot`. */
int moe_b200_import_expert(moe_b200_weights *w, int32_t slot, const void *data, uint64_t bytes);
/* The same, stream-ordered (page-locked data overlaps with other streams; the
 * host buffer must stay valid until the copy completes). */
int moe_b200_import_expert_async(moe_b200_weights *w, int32_t slot, const void *data,
                                 uint64_t bytes, void *stream);
/* Exchanges bank slot `slot` with staging slot `staged` on the device
 * (stream-ordered). Both banks: same device, format and geometry. */
int moe_b200_swap_slots(moe_b200_weights *bank, int32_t slot, moe_b200_weights *staging,
                        int32_t staged, void *stream);

/* Replaces rk_npu_moe_quant_workspace_create / rk_npu_moe_w4_workspace_create
 * (src/npu/moe.rs:200-206). One workspace per stream; reusable by every
 * bank of the same geometry. */
moe_b200_workspace *moe_b200_workspace_create(const moe_b200_config *cfg);
/* Replaces rk_npu_moe_w8_workspace_free. */
void moe_b200_workspace_free(moe_b200_workspace *ws);
/* Replaces rk_npu_moe_w8_workspace_device_bytes. */
uint64_t moe_b200_workspace_device_bytes(const moe_b200_workspace *ws);
/* Moe::max_rows (src/npu/moe.rs:321-323). */
int32_t moe_b200_max_rows(const moe_b200_workspace *ws);

/* Replaces rk_npu_moe_w8_run_f32 (src/npu/moe.rs:372-386): host pointers,
 * synchronous. input [rows][hidden] f32, ids/routes [rows][top], output
 * [rows][hidden] f32 = weighted routed combine (+ shared expert if the bank
 * has one). timings may be NULL. */
int moe_b200_run_f32(moe_b200_workspace *ws, const moe_b200_weights *w, int32_t rows,
                     const float *input, const int32_t *ids, const float *routes,
                     float *output, moe_b200_timings *timings);

/* Extension: same as moe_b200_run_f32 on device pointers, stream-ordered and
 * asynchronous (no host synchronisation). stream is a cudaStream_t. */
int moe_b200_run_device(moe_b200_workspace *ws, const moe_b200_weights *w, int32_t rows,
                        const float *d_input, const int32_t *d_ids, const float *d_routes,
                        float *d_output, void *stream);

/* ---- router-inclusive path (extension; replaces the CPU router of
 * src/model/qwen35/moe.rs:215-241 and the decoder residual add of
 * src/model/qwen35/decoder.rs:215-217) ------------------------------------ */

/* router [experts][hidden] f32 (row e = expert e); bias [experts] f32 added to
 * every logit, or NULL; order MOE_B200_ROUTER_*; min_weight = pruning
 * threshold (src/model/experts/pruning.rs:32-41), 0 = off. */
moe_b200_router *moe_b200_router_create(const moe_b200_config *cfg, const float *router,
                                        const float *bias, int32_t order, float min_weight);
void moe_b200_router_free(moe_b200_router *r);

/* Router options beyond moe_b200_router_create (no counterpart in the
 * reference's native ABI: these replace the CPU-side routing of
 * src/model/ling3tiny/moe.rs:146-223 and the shared-expert gate merge of
 * src/model/qwen35/moe.rs:334-347). */
typedef struct {
    int32_t order;            /* MOE_B200_ROUTER_* */
    int32_t rule;             /* MOE_B200_ROUTE_* */
    float min_weight;         /* softmax rule only: pruning threshold, 0 = off */
    const float *bias;        /* [experts] added to every logit, or NULL */
    /* MOE_B200_ROUTE_GROUPED_SIGMOID (Ling: n_group, topk_group,
     * routed_scaling_factor, gate.expert_bias): score = sigmoid(logit);
     * selected = score + expert_bias; experts / groups >= 2, groups <= 32,
     * top_groups <= groups, top <= top_groups * experts / groups,
     * experts <= 256 */
    int32_t groups, top_groups;
    float routing_scale;
    const float *expert_bias; /* [experts] */
    /* shared-expert gate row [hidden] f32 (mlp.shared_expert_gate.weight), or
     * NULL. With a gate the forward adds sigmoid(gate . x) * shared instead
     * of shared; the gate logit is computed in the router's dot order as
     * one more row after the experts, so router logits have experts + 1
     * columns (the last is the gate logit). */
    const float *shared_gate;
} moe_b200_router_options;

/* Defaults: NEON16 order, softmax rule, no bias, no pruning, no gate. */
void moe_b200_router_options_init(moe_b200_router_options *opt);
/* NULL on an invalid option set. */
moe_b200_router *moe_b200_router_create_ex(const moe_b200_config *cfg, const float *router,
                                           const moe_b200_router_options *opt);

/* Host pointers, synchronous: output = residual + (routed + shared); residual
 * may be NULL. ids/routes, if not NULL, receive the routing [rows][top].
 * With a gated router the shared term is sigmoid(gate . x) * shared.
 * When every buffer given is page-locked (cudaHostAlloc / cudaHostRegister)
 * and no timings are asked for, the workspace captures the call's copies and
 * layer as one CUDA graph and replays it while the buffers (address and
 * allocation), bank, router and row count stay the same; the buffers are read
 * afresh on every call. Pageable buffers run the same kernels eagerly. */
int moe_b200_forward_f32(moe_b200_workspace *ws, const moe_b200_weights *w,
                         const moe_b200_router *r, int32_t rows, const float *input,
                         const float *residual, float *output, int32_t *ids, float *routes,
                         moe_b200_timings *timings);
/* Device pointers, asynchronous on stream. */
int moe_b200_forward_device(moe_b200_workspace *ws, const moe_b200_weights *w,
                            const moe_b200_router *r, int32_t rows, const float *d_input,
                            const float *d_residual, float *d_output, void *stream);

/* ---- stage entry points (extension; for parity checks and expert
 * parallelism). All device pointers, asynchronous. ---------------------- */

/* Router logits (may be NULL; [rows][experts], or [rows][experts + 1] for a
 * router with a shared gate) + the routing rule (top-k, weights, pruning). */
int moe_b200_route_device(moe_b200_workspace *ws, const moe_b200_router *r, int32_t rows,
                          const float *d_input, float *d_logits, int32_t *d_ids,
                          float *d_routes, void *stream);

/* Reads back the workspace's device status word (after synchronising the
 * workspace's last stream) and clears it. Returns 0 or an ERR_DEVICE code. */
int moe_b200_workspace_status(moe_b200_workspace *ws);

/* Device address and size of a workspace buffer, for inspection by tests:
 * "q_x","s_x","perm","pos","offsets","a_perm","s_perm","gate_up" (f32
 * [rows][2I]: dequantised gate then up, before SwiGLU),"q_m","s_m","y",
 * "shared_y","logits" ([rows][experts], or [rows][experts + 1] after a gated
 * router),"ids","routes". Valid until the next call. */
int moe_b200_workspace_buffer(moe_b200_workspace *ws, const char *name, void **d_ptr,
                              uint64_t *bytes);

/* Re-runs one grouped GEMM of the last call in accumulator-dump mode:
 * which = 0 (routed gate/up), 1 (routed down). Writes the raw int32
 * accumulators: per-channel [rows][n], group-32 [rows][k/32][n], rows in the
 * permuted order of "perm". */
int moe_b200_debug_accumulators(moe_b200_workspace *ws, const moe_b200_weights *w,
                                int32_t which, int32_t *d_acc, uint64_t capacity_elems,
                                void *stream);

/* Stage profiling of device-pointer calls (extension). While enabled, every
 * run/forward call records CUDA events between its stages on the launching
 * stream into a ring of 256 slots (slot = call index since enabling); no host
 * synchronisation is added. profile_read synchronises on the slot's last
 * event and fills the stage fields of *t for call `call` (0-based). */
int moe_b200_workspace_profile(moe_b200_workspace *ws, int32_t enable);
int moe_b200_workspace_profile_read(moe_b200_workspace *ws, int32_t call, moe_b200_timings *t);

/* Number of kernels this workspace has launched since creation. */
int64_t moe_b200_workspace_launches(const moe_b200_workspace *ws);

/* ---- CUDA-graph replay (no counterpart in the reference): one router-
 * inclusive device forward of a fixed row count over fixed device buffers,
 * captured once; each replay is a single launch, which removes the host's
 * per-kernel launch cost (the bulk of a decode step). The buffers, weights,
 * router and workspace must outlive the graph; one replay at a time per
 * workspace. --------------------------------------------------------------- */
typedef struct moe_b200_graph moe_b200_graph;
moe_b200_graph *moe_b200_graph_create(moe_b200_workspace *ws, const moe_b200_weights *w,
                                      const moe_b200_router *r, int32_t rows,
                                      const float *d_input, const float *d_residual,
                                      float *d_output);
int moe_b200_graph_launch(moe_b200_graph *g, void *stream);
void moe_b200_graph_free(moe_b200_graph *g);

/* ---- expert parallelism (no counterpart in the reference: its experts run
 * on one device). Rank g of G owns experts [g*P, (g+1)*P), P = experts per
 * rank; the caller moves the packed rows between ranks (NCCL all-to-all) and
 * owns every d_* buffer. Rows are moe_b200_workspace_row_bytes(ws) bytes
 * apart (H rounded up to 256). ---------------------------------------------- */

/* Row stride, in bytes, of the int8 rows the expert-parallel entry points read
 * and write (the workspace's padded hidden size). */
int64_t moe_b200_workspace_row_bytes(const moe_b200_workspace *ws);

/* Token owner, step 1: A8-quantises rows (MoE rule) and packs one int8 row per
 * kept assignment into d_send_q, grouped by destination rank (expert / P) and
 * in assignment order t*k+r within a rank; d_send_scale / d_send_expert get
 * the row's scale and its expert id local to the destination; d_send_counts
 * [world] the rows per destination; d_pos [rows*k] the send slot of each
 * assignment (-1 when pruned). ws: a workspace over all E experts. */
int moe_b200_ep_pack(moe_b200_workspace *ws, int32_t rows, const float *d_x,
                     const int32_t *d_ids, const float *d_routes, int32_t experts_per_rank,
                     int32_t world, int8_t *d_send_q, float *d_send_scale,
                     int32_t *d_send_expert, int32_t *d_send_counts, int32_t *d_pos,
                     void *stream);

/* Expert owner, step 2: the grouped expert FFN (gate/up, SwiGLU, requant,
 * down) of n received rows, expert ids local to w (a bank of P experts);
 * d_y [n][H] f32 in the received order. ws: a workspace over the P experts
 * with max_rows * top >= n. */
int moe_b200_ep_expert_rows(moe_b200_workspace *ws, const moe_b200_weights *w, int32_t n,
                            const int8_t *d_q, const float *d_scale, const int32_t *d_expert,
                            float *d_y, void *stream);

/* Device-initiated exchange over NVLink peer memory (replaces the caller's
 * NCCL all-to-alls and their host-side split sizes). Each rank creates one
 * exchange (up to cap rows from any one source, rows of row_bytes =
 * moe_b200_workspace_row_bytes of the token-side workspace, hidden H),
 * shares its MOE_B200_EP_HANDLE_BYTES handle with the other ranks (any host
 * transport), connects with all world handles in rank order, and then per
 * layer step calls moe_b200_ep_exchange_step after moe_b200_ep_pack: the
 * packed rows go straight into their owners' memory, the owner runs its
 * experts (ws / w: the expert-side workspace with max_rows * top >= world *
 * cap, and the rank's bank), and the expert rows come back into this rank's
 * y_back at the packed positions, ready for moe_b200_ep_combine. No host
 * synchronisation; every wait for a peer gives up after about 2 s with
 * MOE_B200_ERR_DEVICE_TIMEOUT (moe_b200_ep_exchange_status). Every rank
 * must call step the same number of times. */
#define MOE_B200_EP_HANDLE_BYTES 64
typedef struct moe_b200_ep_exchange moe_b200_ep_exchange;
moe_b200_ep_exchange *moe_b200_ep_exchange_create(int32_t device, int32_t world, int32_t rank,
                                                  int32_t cap, int64_t row_bytes, int32_t hidden);
int moe_b200_ep_exchange_handle(const moe_b200_ep_exchange *ex, void *handle);
int moe_b200_ep_exchange_connect(moe_b200_ep_exchange *ex, const void *handles);
int moe_b200_ep_exchange_step(moe_b200_ep_exchange *ex, moe_b200_workspace *ws,
                              const moe_b200_weights *w, const int8_t *d_send_q,
                              const float *d_send_scale, const int32_t *d_send_expert,
                              const int32_t *d_send_counts, void *stream);
/* [cap][hidden] f32: the returned expert rows at this rank's packed positions. */
const float *moe_b200_ep_exchange_y_back(const moe_b200_ep_exchange *ex);
/* Synchronises the device, reads and clears the exchange's status word. */
int moe_b200_ep_exchange_status(moe_b200_ep_exchange *ex);
/* Diagnostics of the failure path (no counterpart in the reference): on a
 * single-rank exchange (world 1), starts a step that no source completes and
 * runs the exchange's row wait on it, which gives up after its limit (about
 * 2 s); the next moe_b200_ep_exchange_status returns
 * MOE_B200_ERR_DEVICE_TIMEOUT, and the exchange and the context stay usable
 * (the next real step completes). MOE_B200_ERR_INVALID for world > 1, where
 * it would break the ranks' lockstep. */
int moe_b200_ep_exchange_probe_timeout(moe_b200_ep_exchange *ex, void *stream);
/* Stage timings of exchange steps (no counterpart in the reference; the
 * exchange-side analogue of moe_b200_workspace_profile): while enabled, each
 * step records CUDA events on its stream; _read waits for the last step and
 * writes its five stage times in microseconds: dispatch (the rows' peer
 * stores), rows wait (until every source's rows arrived), expert rows
 * (grouping, gate/up, requantisation, down), return (the expert rows' peer
 * stores), return wait. MOE_B200_ERR_INVALID before a profiled step. */
int moe_b200_ep_exchange_profile(moe_b200_ep_exchange *ex, int32_t enable);
int moe_b200_ep_exchange_profile_read(moe_b200_ep_exchange *ex, float *stage_us);
void moe_b200_ep_exchange_free(moe_b200_ep_exchange *ex);

/* Token owner, step 3: out[t] = (residual[t] +) sum over ranks r ascending of
 * fma(y_back[pos[t*k+r]], routes[t,r]) for kept assignments, the order of the
 * single-device combine. */
int moe_b200_ep_combine(moe_b200_workspace *ws, int32_t rows, const float *d_y_back,
                        const int32_t *d_pos, const float *d_routes, const float *d_residual,
                        float *d_out, void *stream);

/* Pre-norm of a layer stack: RMSNorm (src/ops/norm.rs:81-106, the norm the
 * decoder applies before each MoE layer, src/model/qwen35/decoder.rs:180-189)
 * of `rows` device rows of `width` floats, on the current device and stream:
 * out[r,i] = (x[r,i] * s_r) * w_i with s_r = 1 / sqrt(sum_i x[r,i]^2 / width +
 * epsilon), the squares summed in column order as the reference's iterator
 * sum, w_i replaced by 1 + w_i when zero_centered. Bit-exact with the
 * reference's f32 arithmetic. d_x and d_out may be the same buffer.
 * MOE_B200_ERR_INVALID for width <= 0 or an epsilon that is not finite and
 * positive (the reference's own checks). */
int moe_b200_rms_norm(const float *d_x, const float *d_weight, int32_t rows, int32_t width,
                      float epsilon, int32_t zero_centered, float *d_out, void *stream);

/* Router + top-k that allocates nothing (no counterpart in the reference; an
 * addition for callers that cannot call cudaMalloc, such as an engine whose
 * own pool owns all device memory, or a hot path that must not risk an
 * allocation or its device synchronisation). Same results as
 * moe_b200_route_device, but without a workspace or router object: the
 * caller passes device input [rows][hidden] f32, router weights
 * [experts][hidden] f32, optional bias [experts] (or NULL), and the device
 * outputs ids / routes [rows][top]. Scratch (logits and tile counters) lives
 * in one fixed device array of the library, about 4.3 MiB on every GPU that
 * loads it, kept until exit; rows * experts must not exceed
 * MOE_B200_NOALLOC_MAX_LOGITS, else MOE_B200_ERR_NOALLOC_LIMIT. Runs on the
 * calling thread's current device (the stream must belong to it). The first
 * call on a device looks up the scratch array's device address, so make that
 * first call before any stream capture. All calls on a device share the
 * scratch: calls that overlap on the GPU (other streams or host threads) race
 * and must be serialised by the caller. Asynchronous; non-finite logits are
 * not reported by this entry point. Checked before anything is launched:
 * hidden % 32 == 0 and, for fewer than 16 rows in the NEON16 order, hidden
 * <= 5664 (the router rows are staged in shared memory), else
 * MOE_B200_ERR_UNSUPPORTED; d_input and d_router 16-byte aligned, d_bias,
 * d_ids and d_routes 4-byte aligned, else MOE_B200_ERR_INVALID. */
#define MOE_B200_NOALLOC_MAX_LOGITS (1 << 20)
int moe_b200_route_noalloc(const float *d_input, const float *d_router, const float *d_bias,
                           int32_t rows, int32_t hidden, int32_t experts, int32_t top,
                           int32_t order, float min_weight, int32_t *d_ids, float *d_routes,
                           void *stream);

/* Replaces rk_npu_strerror (src/npu.rs:187-193). */
const char *moe_b200_strerror(int code);

/* Library build/identity: returns "moe_b200 <version> sm_100a". */
const char *moe_b200_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
