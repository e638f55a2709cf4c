/*
 * CPU restatement of the reference MoE feed-forward path (TEST INFRASTRUCTURE).
 *
 * This library is the parity oracle and the timed CPU baseline for the
 * B200 MoE kernels. Only the tests, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may load it; the product library never does.
 *
 * Every function names the reference file:line whose behaviour it restates
 * (paths relative to the happyme531/open_rknpu2_lm_infer project root).
 * The routed-expert GEMMs of the reference live in an un-vendored submodule
 * (native/rk_npu_matmul), so their arithmetic is restated from the
 * reference's call sites and design notes; parity for those stages is
 * therefore "defined here", and the group-32 fp16 scale format is an
 * extension the reference does not have (its loader rejects group scales,
 * src/model/checkpoint.rs:251-263).
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Router accumulation orders: dense_dot of src/model/cpu.rs:96-153 (NEON16,
 * SEQUENTIAL), and the TF32 NPU linear of src/npu/tf32.rs (TF32). */
enum { ORACLE_ROUTER_NEON16 = 0, ORACLE_ROUTER_SEQUENTIAL = 1, ORACLE_ROUTER_TF32 = 2 };
/* Routing rules: softmax top-k (src/model/qwen35/moe.rs:51-67) and Ling's
 * grouped sigmoid top-k (src/model/ling3tiny/moe.rs:146-223). */
enum { ORACLE_ROUTE_SOFTMAX = 0, ORACLE_ROUTE_GROUPED_SIGMOID = 1 };
/* Activation quantisation rules. */
enum { ORACLE_QUANT_MOE = 0, ORACLE_QUANT_DENSE = 1 };
/* Shared expert modes. */
enum { ORACLE_SHARED_JOINT = 0, ORACLE_SHARED_DENSE = 1 };

/* A quantised matrix in the reference's QuantMatrix layout
 * (src/npu.rs:135-157): codes [k][n] (row k holds the n output channels),
 * per-channel f32 scales [n]; or, when group > 0, fp16 scales [k/group][n]. */
typedef struct {
    int bits;                 /* 4 or 8 */
    int k, n;
    int group;                /* 0 = per output channel, else group size along k */
    const int8_t *codes;      /* [k][n] */
    const float *scales;      /* [n]            (group == 0) */
    const uint16_t *gscales;  /* [k/group][n]   (group > 0), IEEE fp16 bits */
} oracle_qmat;

typedef struct {
    int hidden, inter, experts, top;
    int shared_inter;         /* 0 = no shared expert */
    int shared_mode;          /* ORACLE_SHARED_* */
    int router_order;         /* ORACLE_ROUTER_* */
    float min_weight;         /* pruning threshold, 0 = off */
    const float *router;      /* [experts][hidden] f32 */
    const float *router_bias; /* [experts] added to each logit, or NULL (synthetic skew) */
    const oracle_qmat *gate_up;  /* [experts]: k=hidden, n=2*inter */
    const oracle_qmat *down;     /* [experts]: k=inter,  n=hidden */
    const oracle_qmat *shared_gate_up; /* k=hidden, n=2*shared_inter */
    const oracle_qmat *shared_down;    /* k=shared_inter, n=hidden */
    /* grouped sigmoid routing (route_rule = ORACLE_ROUTE_GROUPED_SIGMOID) */
    int route_rule;
    int groups, top_groups;
    float routing_scale;
    const float *expert_bias; /* [experts] selection bias */
    /* shared-expert gate [hidden] f32 (src/model/qwen35/moe.rs:334-347), or
     * NULL: the shared output is added as sigmoid(gate . x) * shared */
    const float *shared_gate;
} oracle_layer;

/* Optional stage dumps; any pointer may be NULL. Sizes for T tokens, A = number
 * of kept assignments (weight > 0), G_gu = hidden/group, G_d = inter/group. */
typedef struct {
    float *logits;     /* [T][E] */
    int32_t *ids;      /* [T][k] */
    float *weights;    /* [T][k] */
    int32_t *perm;     /* [A] assignment index t*k+r, grouped by expert */
    int32_t *offsets;  /* [E+1] */
    int8_t *qx;        /* [T][H] */
    float *sx;         /* [T] */
    float *middle;     /* [A][I] f32 SwiGLU output, permuted order */
    int8_t *qm;        /* [A][I] */
    float *sm;         /* [A] */
    float *y;          /* [A][H] per-assignment down output, permuted order */
    float *routed;     /* [T][H] weighted combine of routed experts */
    float *shared;     /* [T][H] shared expert output */
    int32_t n_assign;  /* out: A */
    float *shared_scale; /* [T] sigmoid of the shared gate (when the layer has one) */
} oracle_dump;

/* Total-order key of Rust's f32::total_cmp, as a signed integer. */
int32_t oracle_total_key(float v);

void oracle_router_logits(const float *x, const float *router, const float *bias, int T,
                          int H, int E, int order, float *logits);
int oracle_routes(const float *logits, int T, int E, int k, float min_weight,
                  int32_t *ids, float *weights);
int oracle_ling_routes(const float *logits, const float *bias, int T, int E, int groups,
                       int top_groups, int k, float routing_scale, int32_t *ids,
                       float *weights);
float oracle_sigmoid(float x);
int oracle_permute(const int32_t *ids, const float *weights, int T, int k, int E,
                   int32_t *perm, int32_t *offsets);
void oracle_quantize(const float *x, int rows, int cols, int rule, int8_t *q, float *s);
void oracle_gemm_acc(const int8_t *q, int rows, const oracle_qmat *w, int32_t *acc);
void oracle_gemm_dequant(const int8_t *q, const float *s, int rows, const oracle_qmat *w,
                         float *out);
void oracle_swiglu(const float *gu, int rows, int width, float *out);
void oracle_rms_norm(const float *x, const float *weight, int rows, int width, float eps,
                     int zero_centered, float *out);
int oracle_moe_run(const oracle_layer *L, int T, const float *x, const int32_t *ids,
                   const float *weights, float *out, oracle_dump *dump);
int oracle_moe_forward(const oracle_layer *L, int T, const float *x, const float *residual,
                       float *out, oracle_dump *dump);
float oracle_half_to_float(uint16_t h);
uint16_t oracle_float_to_half(float f);
int oracle_threads(void);

#ifdef __cplusplus
}
#endif
#endif
