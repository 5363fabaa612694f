/*
 * noor_oracle.c -- CPU restatement of Noor's sparse-MoE layer forward.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in noor_-_bangla_ai_b200/csrc: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference leg may load it.  The product
 * path never calls into it.
 *
 * It restates, step by step, the f32 host path of the Rust crate noor-core
 * (Adiuk24/Noor_-_Bangla_AI):
 *
 *   crates/noor-core/src/layers/moe.rs:79-107    MoERouter::route
 *   crates/noor-core/src/layers/moe.rs:40-45     ExpertUtilization::record
 *   crates/noor-core/src/layers/moe.rs:145-177   MoELayer::forward
 *   crates/noor-core/src/layers/ffn.rs:24-34     GeGLUFFN::forward  (dense branch)
 *   crates/noor-core/src/layers/ffn.rs:62-68     SwiGLUFFN::forward (experts)
 *   crates/noor-core/src/layers/parallel_ffn.rs:30-36  ParallelFFN::forward
 *   crates/noor-core/src/tensor.rs:23-33         f32_to_bf16 / bf16_to_f32 (RNE)
 *   crates/noor-core/src/tensor.rs:280-299       add / mul
 *   crates/noor-core/src/tensor.rs:428-459       sigmoid / gelu (tanh) / silu
 *   crates/noor-core/src/tensor.rs:462-490       rms_norm (f64 accumulation)
 *   crates/noor-core/src/kernels.rs:151-163      cblas_sgemm row-major, beta = 0
 *   crates/noor-train/src/optim/smebu.rs:36-48   SMEBU::update
 *
 * Build: -O2 -ffp-contract=off so that every f32 multiply and add rounds
 * separately, as Rust emits them (Rust never contracts a*b+c into an FMA).
 * expf/tanhf come from glibc's libm, which is what Rust's f32::exp / f32::tanh
 * call on Linux.
 *
 * Parity pinning: the reference's own tests hold no golden tensors for the MoE
 * path (its RNG is unseeded, tensor.rs:129-140).  This restatement is pinned
 * against every known-answer test the reference has on this path (matmul
 * 2x2 / ones / 128x64x96, sigmoid, silu, gelu, BF16 RNE, SMEBU, the router
 * structural tests, utilization sums, parameter counts): see
 * tests/test_oracle.py and tests/golden/.  The full-layer numerics are
 * cross-checked against an independent numpy restatement (oracle/oracle.py).
 *
 * The matmul goes either to a plain loop (k ascending per output element,
 * the accumulation order of tensor.rs:351-382) or, for timing the
 * reference-faithful CPU baseline, to OpenBLAS sgemm loaded with dlopen
 * (the cblas route the reference takes on x86, kernels.rs:151-163).
 */
#include <dlfcn.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* BF16 storage rounding: tensor.rs:23-33                                    */
/* ------------------------------------------------------------------------ */

uint16_t noor_oracle_f32_to_bf16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    uint32_t rounding_bias = ((bits >> 16) & 1u) + 0x7FFFu;
    return (uint16_t)((bits + rounding_bias) >> 16); /* wrapping add */
}

float noor_oracle_bf16_to_f32(uint16_t h) {
    uint32_t bits = ((uint32_t)h) << 16;
    float x;
    memcpy(&x, &bits, 4);
    return x;
}

/* Round every element to the nearest BF16 value (kept as f32), in place. */
void noor_oracle_round_bf16(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = noor_oracle_bf16_to_f32(noor_oracle_f32_to_bf16(x[i]));
}

/* ------------------------------------------------------------------------ */
/* Elementwise ops: tensor.rs:280-299, 428-459                              */
/* ------------------------------------------------------------------------ */

float noor_oracle_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

float noor_oracle_silu(float x) { return x / (1.0f + expf(-x)); }

float noor_oracle_gelu(float x) {
    /* sqrt_2_pi = (2.0f32 / PI).sqrt(); inner = sqrt_2_pi * (x + 0.044715*x*x*x);
     * 0.5 * x * (1.0 + inner.tanh()) -- every literal is f32 in the Rust source. */
    const float sqrt_2_pi = sqrtf(2.0f / 3.14159265358979323846f);
    float cube = 0.044715f * x;
    cube = cube * x;
    cube = cube * x;
    float inner = sqrt_2_pi * (x + cube);
    float half_x = 0.5f * x;
    return half_x * (1.0f + tanhf(inner));
}

/* ------------------------------------------------------------------------ */
/* Matmul boundary: kernels.rs:141-184 (cblas_sgemm, beta = 0 => overwrite)   */
/* ------------------------------------------------------------------------ */

typedef void (*sgemm64_fn)(int order, int ta, int tb, int64_t m, int64_t n, int64_t k, float alpha,
                           const float* a, int64_t lda, const float* b, int64_t ldb, float beta,
                           float* c, int64_t ldc);
typedef void (*set_threads_fn)(int);

static sgemm64_fn g_sgemm = 0;
static set_threads_fn g_set_threads = 0;

/* Route matmuls to an ILP64 OpenBLAS (numpy's bundled scipy_openblas64_).
 * Returns 0 on success; path NULL switches back to the plain loop. */
int noor_oracle_use_openblas(const char* path, int threads) {
    if (!path) {
        g_sgemm = 0;
        return 0;
    }
    void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) return 1;
    g_sgemm = (sgemm64_fn)dlsym(h, "scipy_cblas_sgemm64_");
    g_set_threads = (set_threads_fn)dlsym(h, "scipy_goto_set_num_threads64_");
    if (!g_sgemm) return 2;
    if (g_set_threads && threads > 0) g_set_threads(threads);
    return 0;
}

/* C[m,n] = A[m,k] . B[k,n], row-major, C overwritten. */
void noor_oracle_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n) {
    if (g_sgemm) {
        g_sgemm(101, 111, 111, m, n, k, 1.0f, a, k, b, n, 0.0f, c, n);
        return;
    }
    memset(c, 0, (size_t)(m * n) * sizeof(float));
    for (int64_t i = 0; i < m; ++i) {
        float* crow = c + i * n;
        for (int64_t kk = 0; kk < k; ++kk) {
            const float av = a[i * k + kk];
            const float* brow = b + kk * n;
            for (int64_t j = 0; j < n; ++j) crow[j] += av * brow[j];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Router: moe.rs:79-107                                                    */
/* ------------------------------------------------------------------------ */

/* scores[E] scratch.  idx/w receive min(k,E) entries in rank order. */
static void route_one(const float* x, const float* gate, const float* bias, const float* scales,
                      int64_t d, int64_t ne, int64_t k, float* scores, int32_t* order,
                      int32_t* idx, float* w) {
    for (int64_t e = 0; e < ne; ++e) {
        float dot = 0.0f;
        for (int64_t i = 0; i < d; ++i) dot += x[i] * gate[i * ne + e];
        dot += bias[e];
        scores[e] = 1.0f / (1.0f + expf(-dot));
    }
    /* indexed.sort_by(|a,b| b.1.partial_cmp(&a.1)) is a stable descending
     * sort: equal scores keep ascending expert order.  Insertion sort with a
     * strict comparison is stable. */
    for (int64_t e = 0; e < ne; ++e) order[e] = (int32_t)e;
    for (int64_t i = 1; i < ne; ++i) {
        int32_t cur = order[i];
        int64_t j = i - 1;
        while (j >= 0 && scores[order[j]] < scores[cur]) {
            order[j + 1] = order[j];
            --j;
        }
        order[j + 1] = cur;
    }
    int64_t kk = k < ne ? k : ne;
    for (int64_t r = 0; r < kk; ++r) {
        idx[r] = order[r];
        w[r] = scores[order[r]] * scales[order[r]];
    }
}

/* Route T tokens.  idx/w are [T,k]; counts[E] is ADDED to (record, moe.rs:40-45);
 * scores_out, if non-null, receives the f32 sigmoid scores [T,E]. */
void noor_oracle_route(const float* x, const float* gate, const float* bias, const float* scales,
                       int64_t T, int64_t d, int64_t ne, int64_t k, int32_t* idx, float* w,
                       int64_t* counts, float* scores_out) {
    float* scores = (float*)malloc(sizeof(float) * ne);
    int32_t* order = (int32_t*)malloc(sizeof(int32_t) * ne);
    int64_t kk = k < ne ? k : ne;
    for (int64_t t = 0; t < T; ++t) {
        route_one(x + t * d, gate, bias, scales, d, ne, k, scores, order, idx + t * kk, w + t * kk);
        if (counts)
            for (int64_t r = 0; r < kk; ++r) counts[idx[t * kk + r]] += 1;
        if (scores_out) memcpy(scores_out + t * ne, scores, sizeof(float) * ne);
    }
    free(scores);
    free(order);
}

/* f64 restatement of the router scores, for classifying near-ties: the exact
 * dot (accumulated in double), its running absolute sum (for an error bound),
 * and the double sigmoid. */
void noor_oracle_scores_f64(const float* x, const float* gate, const float* bias, int64_t T,
                            int64_t d, int64_t ne, double* scores, double* abs_dot) {
    for (int64_t t = 0; t < T; ++t) {
        const float* xr = x + t * d;
        for (int64_t e = 0; e < ne; ++e) {
            double dot = 0.0, ab = 0.0;
            for (int64_t i = 0; i < d; ++i) {
                double p = (double)xr[i] * (double)gate[i * ne + e];
                dot += p;
                ab += fabs(p);
            }
            dot += (double)bias[e];
            scores[t * ne + e] = 1.0 / (1.0 + exp(-dot));
            if (abs_dot) abs_dot[t * ne + e] = ab + fabs((double)bias[e]);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* FFNs: ffn.rs:24-34 (GeGLU) and ffn.rs:62-68 (SwiGLU)                      */
/* ------------------------------------------------------------------------ */

/* act: 0 = GELU (tanh form), 1 = SiLU.  x[m,d] -> out[m,d]; weights are the
 * reference layout: w_gate [d,ff], w_up [d,ff], w_down [ff,d]. */
void noor_oracle_glu_ffn(const float* x, int64_t m, int64_t d, int64_t ff, const float* w_gate,
                         const float* w_up, const float* w_down, int act, float* out) {
    float* gate = (float*)malloc(sizeof(float) * m * ff);
    float* up = (float*)malloc(sizeof(float) * m * ff);
    noor_oracle_matmul(x, w_gate, gate, m, d, ff);
    noor_oracle_matmul(x, w_up, up, m, d, ff);
    for (int64_t i = 0; i < m * ff; ++i) {
        float a = act == 0 ? noor_oracle_gelu(gate[i]) : noor_oracle_silu(gate[i]);
        gate[i] = a * up[i]; /* tensor::mul */
    }
    noor_oracle_matmul(gate, w_down, out, m, ff, d);
    free(gate);
    free(up);
}

/* ------------------------------------------------------------------------ */
/* MoELayer::forward (moe.rs:145-177)                                       */
/* ------------------------------------------------------------------------ */

typedef struct {
    int64_t d_model, n_experts, top_k, expert_ff, dense_ff;
    const float* gate;   /* [d,E] */
    const float* bias;   /* [E]   */
    const float* scales; /* [E]   */
    const float* w_gate; /* [E,d,ff] (expert e at e*d*ff) */
    const float* w_up;   /* [E,d,ff] */
    const float* w_down; /* [E,ff,d] */
    const float* shared_gate, *shared_up, *shared_down; /* nullable: [d,ff],[d,ff],[ff,d] */
    const float* dense_gate, *dense_up, *dense_down;    /* [d,dff],[d,dff],[dff,d] */
} noor_oracle_layer;

/* out[T,d] = MoELayer::forward(x).  idx/w [T,k] and counts[E] (added to) are
 * optional outputs of the router. */
void noor_oracle_moe_forward(const noor_oracle_layer* L, const float* x, int64_t T, float* out,
                             int32_t* idx_out, float* w_out, int64_t* counts) {
    const int64_t d = L->d_model, ne = L->n_experts, ff = L->expert_ff;
    const int64_t kk = L->top_k < ne ? L->top_k : ne;
    float* scores = (float*)malloc(sizeof(float) * ne);
    int32_t* order = (int32_t*)malloc(sizeof(int32_t) * ne);
    int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * kk);
    float* w = (float*)malloc(sizeof(float) * kk);
    float* y = (float*)malloc(sizeof(float) * d);
    memset(out, 0, sizeof(float) * T * d);
    for (int64_t s = 0; s < T; ++s) {
        const float* tok = x + s * d;
        route_one(tok, L->gate, L->bias, L->scales, d, ne, kk, scores, order, idx, w);
        if (counts)
            for (int64_t r = 0; r < kk; ++r) counts[idx[r]] += 1;
        if (idx_out) memcpy(idx_out + s * kk, idx, sizeof(int32_t) * kk);
        if (w_out) memcpy(w_out + s * kk, w, sizeof(float) * kk);
        float* o = out + s * d;
        for (int64_t r = 0; r < kk; ++r) {
            const int64_t e = idx[r];
            noor_oracle_glu_ffn(tok, 1, d, ff, L->w_gate + e * d * ff, L->w_up + e * d * ff,
                                L->w_down + e * ff * d, 1, y);
            const float wt = w[r];
            for (int64_t j = 0; j < d; ++j) o[j] += wt * y[j];
        }
        if (L->shared_gate) {
            noor_oracle_glu_ffn(tok, 1, d, ff, L->shared_gate, L->shared_up, L->shared_down, 1, y);
            for (int64_t j = 0; j < d; ++j) o[j] += y[j];
        }
    }
    free(scores);
    free(order);
    free(idx);
    free(w);
    free(y);
}

/* ParallelFFN::forward (parallel_ffn.rs:30-36): (dense(x) + moe(x)) * (1/sqrt 2). */
void noor_oracle_parallel_forward(const noor_oracle_layer* L, const float* x, int64_t T, float* out,
                                  int32_t* idx_out, float* w_out, int64_t* counts) {
    const int64_t d = L->d_model;
    float* dense = (float*)malloc(sizeof(float) * T * d);
    noor_oracle_glu_ffn(x, T, d, L->dense_ff, L->dense_gate, L->dense_up, L->dense_down, 0, dense);
    noor_oracle_moe_forward(L, x, T, out, idx_out, w_out, counts);
    const float inv_sqrt2 = 1.0f / sqrtf(2.0f);
    for (int64_t i = 0; i < T * d; ++i) {
        float c = dense[i] + out[i]; /* tensor::add(dense, moe) */
        out[i] = c * inv_sqrt2;      /* Tensor::scale */
    }
    free(dense);
}

/* ------------------------------------------------------------------------ */
/* rms_norm (tensor.rs:462-490) and SMEBU::update (smebu.rs:36-48)            */
/* ------------------------------------------------------------------------ */

void noor_oracle_rms_norm(const float* a, const float* weight, int64_t n_vecs, int64_t dim, double eps,
                          float* out) {
    for (int64_t v = 0; v < n_vecs; ++v) {
        const float* row = a + v * dim;
        double sum_sq = 0.0;
        for (int64_t i = 0; i < dim; ++i) {
            double val = (double)row[i];
            sum_sq += val * val;
        }
        double rms = sqrt(sum_sq / (double)dim + eps);
        for (int64_t i = 0; i < dim; ++i)
            out[v * dim + i] = (float)((double)row[i] / rms * (double)weight[i]);
    }
}

void noor_oracle_smebu_update(float* momentum, float* biases, const float* fractions, int64_t ne,
                              float kappa, float beta, float lambda) {
    const float f_target = 1.0f / (float)ne;
    for (int64_t i = 0; i < ne; ++i) {
        momentum[i] = beta * momentum[i] + lambda * (f_target - fractions[i]);
        biases[i] = kappa * tanhf(momentum[i] / kappa);
    }
}
