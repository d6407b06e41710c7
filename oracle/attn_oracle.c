/*
 * CPU oracle for haelixe's fused attention path: a C restatement of the
 * reference's own CPU math (the crate is Rust + WGSL and cannot be built
 * or run in this environment).
 *
 * TEST INFRASTRUCTURE ONLY. Only the test-suite, the smoke check and the
 * CPU-baseline leg of the benchmark load this library; the product library
 * (haelixe_b200/csrc) never links or calls it.
 *
 * What it restates (paths inside the reference project):
 *   - forward  : src/ops/flash_attention.rs:18-19 (scores = scale Q K^T,
 *                softmax) + src/gpu/shaders/flash_attention.wgsl:19-123
 *                (same math as an online softmax), O = P V;
 *   - backward : src/ops/flash_attention.rs:16-39 with
 *                src/kernels/activations.rs:154-188 (softmax Jacobian);
 *   - matmul   : src/kernels/matmul.rs:31-126 (64^3 blocks, i-p-j order);
 *   - softmax  : src/kernels/activations.rs:102-152 / softmax.rs:20-44;
 *   - RoPE     : src/kernels/rope.rs:5-82 (interleaved pairs);
 *   - bf16     : round-to-nearest-even, the rounding of `half::bf16::from_f32`
 *                (half 2.7.1, used at src/tensor.rs:706).
 * Deliberate departures (each a defect of the reference, noted in the
 * functions): true transposes instead of the stride-ignoring CPU matmul,
 * dQ/dK multiplied by `scale` (switch `ref_compat` off), and a causal mask.
 *
 * Parity status: PARTIALLY PINNED. The softmax forward/backward kernels are
 * pinned to the reference's golden vectors (haelixe-lab/src/main.rs:35-209)
 * and finite-difference tolerances (tests/tensor_tests.rs:120-190). The
 * reference has no attention test and no runnable attention path, so the
 * attention outputs and gradients themselves are pinned only by the
 * composition of those kernels, by finite differences and by an independent
 * f64 evaluation of the same formulas.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define ORA_BLOCK 64 /* src/kernels/matmul.rs:6-8 */

static int g_threads = 0;

void ora_set_threads(int n) { g_threads = n; }

int ora_num_threads(void) {
    if (g_threads > 0) return g_threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef void (*ora_task_fn)(void* ctx, long begin, long end);

typedef struct {
    ora_task_fn fn;
    void* ctx;
    long begin, end;
} ora_job;

static void* ora_worker(void* arg) {
    ora_job* j = (ora_job*)arg;
    if (j->begin < j->end) j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

/* Split [0, n) into one contiguous chunk per thread (the rayon pool of the
 * reference also defaults to one worker per core). */
static void ora_parallel_for(long n, ora_task_fn fn, void* ctx) {
    int t = ora_num_threads();
    if (t > n) t = (int)n;
    if (t <= 1) {
        if (n > 0) fn(ctx, 0, n);
        return;
    }
    pthread_t th[512];
    ora_job jobs[512];
    if (t > 512) t = 512;
    const long chunk = (n + t - 1) / t;
    for (int i = 0; i < t; ++i) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].begin = i * chunk;
        jobs[i].end = (i + 1) * chunk < n ? (i + 1) * chunk : n;
    }
    for (int i = 1; i < t; ++i) pthread_create(&th[i], NULL, ora_worker, &jobs[i]);
    ora_worker(&jobs[0]);
    for (int i = 1; i < t; ++i) pthread_join(th[i], NULL);
}

/* f32 restatement (the "port"). */
#define REAL float
#define SFX
#define ORA_EXP expf
#define ORA_LOG logf
#include "attn_oracle_impl.h"
#undef REAL
#undef SFX
#undef ORA_EXP
#undef ORA_LOG

/* f64 evaluation of the same formulas (cross-check of the port). */
#define REAL double
#define SFX _f64
#define ORA_EXP exp
#define ORA_LOG log
#include "attn_oracle_impl.h"
#undef REAL
#undef SFX
#undef ORA_EXP
#undef ORA_LOG

/* Row softmax over `rows` rows of length n (out of place), exported for the
 * golden-vector checks of the reference's softmax kernel. */
void ora_softmax(const float* x, float* y, long rows, long n) {
    memcpy(y, x, sizeof(float) * rows * n);
    softmax_rows_inplace(y, NULL, rows, n);
}

/* softmax_backward(dy, y) -> dx, src/kernels/activations.rs:154-188. */
void ora_softmax_backward(const float* dy, const float* y, float* dx, long rows, long n) {
    memcpy(dx, dy, sizeof(float) * rows * n);
    softmax_backward_inplace(dx, y, rows, n);
}

/* RoPE forward, src/kernels/rope.rs:5-44. x is [tokens, D] with the
 * sequence position m = token % S (rope.rs:24); pairs (2i, 2i+1) rotate by
 * theta = m * base^(-(2i)/D) computed in f32 with powf/cosf/sinf
 * (rope.rs:28-31), one multiply and one add/sub per term (rope.rs:37-38). */
void ora_rope_fwd(const float* x, float* out, long tokens, int S, int D, float base) {
    for (long t = 0; t < tokens; ++t) {
        const float m = (float)(t % S);
        const long off = t * D;
        for (int i = 0; i < D / 2; ++i) {
            const float exponent = -((float)(2 * i)) / (float)D;
            const float theta = m * powf(base, exponent);
            const float c = cosf(theta), s = sinf(theta);
            const float x0 = x[off + 2 * i], x1 = x[off + 2 * i + 1];
            const float a = x0 * c, b = x1 * s, e = x0 * s, f = x1 * c;
            out[off + 2 * i] = a - b;
            out[off + 2 * i + 1] = e + f;
        }
    }
}

/* RoPE backward, src/kernels/rope.rs:46-82: the same rotation by -theta
 * (rope.rs:67). */
void ora_rope_bwd(const float* g, float* out, long tokens, int S, int D, float base) {
    for (long t = 0; t < tokens; ++t) {
        const float m = (float)(t % S);
        const long off = t * D;
        for (int i = 0; i < D / 2; ++i) {
            const float exponent = -((float)(2 * i)) / (float)D;
            const float theta = -(m * powf(base, exponent));
            const float c = cosf(theta), s = sinf(theta);
            const float g0 = g[off + 2 * i], g1 = g[off + 2 * i + 1];
            const float a = g0 * c, b = g1 * s, e = g0 * s, f = g1 * c;
            out[off + 2 * i] = a - b;
            out[off + 2 * i + 1] = e + f;
        }
    }
}

/* f32 -> bf16 -> f32 with round-to-nearest-even; NaN stays NaN. */
void ora_round_bf16(const float* x, float* y, long n) {
    for (long i = 0; i < n; ++i) {
        uint32_t u;
        memcpy(&u, &x[i], 4);
        if ((u & 0x7fffffffu) > 0x7f800000u) {
            u = (u | 0x00400000u) & 0xffff0000u;
        } else {
            u += 0x7fffu + ((u >> 16) & 1u);
            u &= 0xffff0000u;
        }
        memcpy(&y[i], &u, 4);
    }
}

/* Row-major out[m, n] = a[m, k] b[k, n]: the blocked i-p-j loop of
 * src/kernels/matmul.rs:95-125 (Tensor::matmul on the CPU, used by
 * Linear::forward, src/nn/linear.rs:55, and by its backward). */
void ora_matmul(const float* a, const float* b, float* out, long m, long k, long n) {
    matmul(a, b, out, m, k, n);
}

/* RMSNorm forward, src/kernels/rms_norm.rs:20-55: per row of `hidden`,
 * sum_sq accumulated in order, inv_rms = 1 / sqrt(sum_sq / hidden + eps),
 * out = x * inv_rms * w. */
void ora_rms_norm_fwd(const float* x, const float* w, float* out, long rows, int hidden, float eps) {
    for (long i = 0; i < rows; ++i) {
        const float* xr = x + i * hidden;
        float* yr = out + i * hidden;
        float sum_sq = 0.0f;
        for (int j = 0; j < hidden; ++j) sum_sq += xr[j] * xr[j];
        const float inv_rms = 1.0f / sqrtf(sum_sq / (float)hidden + eps);
        for (int j = 0; j < hidden; ++j) yr[j] = xr[j] * inv_rms * w[j];
    }
}

/* RMSNorm backward, src/kernels/rms_norm.rs:57-132: inv_rms recomputed, then
 * dot = sum g w x, dx = g w inv_rms - x inv_rms^3 dot / hidden and
 * dw += g x inv_rms, summed over the rows in row order. */
void ora_rms_norm_bwd(const float* g, const float* x, const float* w, float* dx, float* dw, long rows,
                      int hidden, float eps) {
    for (int j = 0; j < hidden; ++j) dw[j] = 0.0f;
    for (long i = 0; i < rows; ++i) {
        const float* gr = g + i * hidden;
        const float* xr = x + i * hidden;
        float* dxr = dx + i * hidden;
        float sum_sq = 0.0f;
        for (int j = 0; j < hidden; ++j) sum_sq += xr[j] * xr[j];
        const float inv_rms = 1.0f / sqrtf(sum_sq / (float)hidden + eps);
        float dot = 0.0f;
        for (int j = 0; j < hidden; ++j) dot += gr[j] * w[j] * xr[j];
        const float inv3 = inv_rms * inv_rms * inv_rms;
        for (int j = 0; j < hidden; ++j) {
            dxr[j] = (gr[j] * w[j] * inv_rms) - (xr[j] * inv3 * dot / (float)hidden);
            dw[j] += gr[j] * xr[j] * inv_rms;
        }
    }
}

/* GELU, tanh form, src/kernels/activations.rs:192-209:
 * c = sqrt(2/pi), inner = c (x + 0.044715 x^3), y = 0.5 x (1 + tanh(inner)). */
void ora_gelu_fwd(const float* x, float* y, long n) {
    const float c = sqrtf(2.0f / 3.14159265358979323846f) /* std::f32::consts::PI */;
    for (long i = 0; i < n; ++i) {
        const float v = x[i];
        const float inner = c * (v + 0.044715f * (v * v * v));
        y[i] = 0.5f * v * (1.0f + tanhf(inner));
    }
}

/* Its derivative times g, activations.rs:211-237:
 * sech2 = 1 - tanh^2, d_inner = c (1 + 3 * 0.044715 x^2),
 * dx = g (0.5 (1 + tanh) + 0.5 x sech2 d_inner). */
void ora_gelu_bwd(const float* g, const float* x, float* dx, long n) {
    const float c = sqrtf(2.0f / 3.14159265358979323846f) /* std::f32::consts::PI */;
    for (long i = 0; i < n; ++i) {
        const float v = x[i];
        const float inner = c * (v + 0.044715f * (v * v * v));
        const float t = tanhf(inner);
        const float sech2 = 1.0f - t * t;
        const float d_inner = c * (1.0f + 3.0f * 0.044715f * (v * v));
        dx[i] = g[i] * (0.5f * (1.0f + t) + 0.5f * v * sech2 * d_inner);
    }
}

/* Cross-entropy forward, src/kernels/loss.rs:46-82: per row the max, the sum
 * of exp(x - max), lse = ln(sum) + max, loss = lse - x[target]; probs =
 * exp(x - max) / sum; returns the mean of the row losses. Targets must be
 * < classes (the reference panics otherwise). */
float ora_cross_entropy_fwd(const float* logits, const uint32_t* targets, float* probs, long rows, long classes) {
    float total = 0.0f;
    for (long r = 0; r < rows; ++r) {
        const float* row = logits + r * classes;
        float mx = -INFINITY;
        for (long j = 0; j < classes; ++j) mx = fmaxf(mx, row[j]);
        float sum = 0.0f;
        for (long j = 0; j < classes; ++j) sum += expf(row[j] - mx);
        const float lse = logf(sum) + mx;
        total += -row[targets[r]] + lse;
        for (long j = 0; j < classes; ++j) probs[r * classes + j] = expf(row[j] - mx) / sum;
    }
    return total / (float)rows;
}

/* Cross-entropy backward, loss.rs:86-117: (probs - onehot) * (1 / rows). */
void ora_cross_entropy_bwd(const float* probs, const uint32_t* targets, float* grads, long rows, long classes) {
    const float scale = 1.0f / (float)rows;
    for (long r = 0; r < rows; ++r)
        for (long j = 0; j < classes; ++j) {
            float g = probs[r * classes + j];
            if ((uint32_t)j == targets[r]) g -= 1.0f;
            grads[r * classes + j] = g * scale;
        }
}

/* f32 a^n, n >= 0, by square-and-multiply: how Rust's f32::powi with a
 * run-time exponent evaluates (llvm.powi). */
static float powi_f32(float a, int n) {
    float r = 1.0f;
    for (;;) {
        if (n & 1) r *= a;
        n /= 2;
        if (n == 0) break;
        a *= a;
    }
    return r;
}

/* AdamW::step for one tensor, src/optim.rs:128-191, with `step` the
 * step_count after the increment at optim.rs:130. */
void ora_adamw_step(float* p, const float* g, float* m, float* v, long n, float lr, float beta1, float beta2,
                    float eps, float weight_decay, int step) {
    const float bc1 = 1.0f - powi_f32(beta1, step);
    const float bc2 = 1.0f - powi_f32(beta2, step);
    for (long i = 0; i < n; ++i) {
        p[i] -= lr * weight_decay * p[i];
        m[i] = beta1 * m[i] + (1.0f - beta1) * g[i];
        v[i] = beta2 * v[i] + (1.0f - beta2) * g[i] * g[i];
        const float m_hat = m[i] / bc1;
        const float v_hat = v[i] / bc2;
        p[i] -= lr * m_hat / (sqrtf(v_hat) + eps);
    }
}
