/*
 * Type-generic body of the CPU attention oracle. Included twice by
 * attn_oracle.c: once with REAL=float (the restatement of the reference's
 * f32 CPU kernels, "port") and once with REAL=double (a higher-precision
 * cross-check of the port itself). SFX names the exported symbol suffix.
 *
 * TEST INFRASTRUCTURE ONLY: nothing in the product library links this code.
 */

#define CAT_(a, b) a##b
#define CAT(a, b) CAT_(a, b)
#define FN(name) CAT(name, SFX)

/* ---- blocked matmul: out[m,n] = a[m,k] . b[k,n] --------------------------
 * Follows src/kernels/matmul.rs:31-126 of the reference: the output starts
 * at zero (matmul.rs:184-185), 64x64x64 blocks (matmul.rs:6-8), parallel
 * over M-blocks (matmul.rs:91), and the i-p-j loop order inside a block
 * (matmul.rs:103-123) with one multiply and one add per term (no FMA).
 * Operands are dense row-major; every transpose is materialised by the
 * caller first, so the stride-ignoring defect of the reference's CPU path
 * (matmul.rs:107-118 indexes i*k and p*n regardless of strides) is not
 * reproduced. */
typedef struct {
    const REAL* a;
    const REAL* b;
    REAL* out;
    long m, k, n;
    int accumulate; /* 1: add onto `out` instead of starting from zero */
} FN(mm_ctx);

static void FN(mm_task)(void* vctx, long bm0, long bm1) {
    FN(mm_ctx)* c = (FN(mm_ctx)*)vctx;
    const long m = c->m, k = c->k, n = c->n;
    for (long bm = bm0; bm < bm1; ++bm) {
        const long m_start = bm * ORA_BLOCK;
        const long m_end = (m_start + ORA_BLOCK) < m ? (m_start + ORA_BLOCK) : m;
        if (!c->accumulate) {
            for (long i = m_start; i < m_end; ++i) {
                REAL* row = c->out + i * n;
                for (long j = 0; j < n; ++j) row[j] = (REAL)0;
            }
        }
        for (long n_start = 0; n_start < n; n_start += ORA_BLOCK) {
            const long n_end = (n_start + ORA_BLOCK) < n ? (n_start + ORA_BLOCK) : n;
            for (long k_start = 0; k_start < k; k_start += ORA_BLOCK) {
                const long k_end = (k_start + ORA_BLOCK) < k ? (k_start + ORA_BLOCK) : k;
                for (long i = m_start; i < m_end; ++i) {
                    REAL* c_row = c->out + i * n;
                    const REAL* a_row = c->a + i * k;
                    for (long p = k_start; p < k_end; ++p) {
                        const REAL a_val = a_row[p];
                        const REAL* b_row = c->b + p * n;
                        for (long j = n_start; j < n_end; ++j) {
                            c_row[j] = c_row[j] + a_val * b_row[j];
                        }
                    }
                }
            }
        }
    }
}

static void FN(matmul)(const REAL* a, const REAL* b, REAL* out, long m, long k, long n) {
    FN(mm_ctx) c = {a, b, out, m, k, n, 0};
    ora_parallel_for((m + ORA_BLOCK - 1) / ORA_BLOCK, FN(mm_task), &c);
}

/* out += a . b, with each output element's terms added in the same k order
 * as `matmul` (used to sum a product over consecutive row blocks of k). */
static void FN(matmul_acc)(const REAL* a, const REAL* b, REAL* out, long m, long k, long n) {
    FN(mm_ctx) c = {a, b, out, m, k, n, 1};
    ora_parallel_for((m + ORA_BLOCK - 1) / ORA_BLOCK, FN(mm_task), &c);
}

/* ---- scalar multiply (src/kernels/activations.rs:87-100, `scalar_mul`) -- */
static void FN(scale_inplace)(REAL* x, long n, REAL s) {
    for (long i = 0; i < n; ++i) x[i] = x[i] * s;
}

/* ---- dense transpose, out[c,r] = in[r,c] ------------------------------- */
typedef struct {
    const REAL* in;
    REAL* out;
    long rows, cols;
} FN(tr_ctx);

static void FN(tr_task)(void* vctx, long r0, long r1) {
    FN(tr_ctx)* c = (FN(tr_ctx)*)vctx;
    for (long r = r0; r < r1; ++r)
        for (long col = 0; col < c->cols; ++col) c->out[col * c->rows + r] = c->in[r * c->cols + col];
}

static void FN(transpose)(const REAL* in, REAL* out, long rows, long cols) {
    FN(tr_ctx) c = {in, out, rows, cols};
    ora_parallel_for(rows, FN(tr_task), &c);
}

/* ---- row softmax (src/kernels/activations.rs:102-152; the same math as
 * src/kernels/softmax.rs:20-44): max, exp(x - max) with a running f32 sum,
 * then divide by the sum. Rows whose entries are all -inf never occur here
 * (the causal mask always keeps the diagonal). `lse` (optional) receives
 * max + log(sum), which the reference does not produce; the CUDA path
 * stores it for the backward. --------------------------------------------- */
typedef struct {
    REAL* x;
    float* lse;
    long n;
} FN(sm_ctx);

static void FN(sm_task)(void* vctx, long r0, long r1) {
    FN(sm_ctx)* c = (FN(sm_ctx)*)vctx;
    const long n = c->n;
    for (long r = r0; r < r1; ++r) {
        REAL* row = c->x + r * n;
        REAL max_val = -(REAL)INFINITY;
        for (long i = 0; i < n; ++i)
            if (row[i] > max_val) max_val = row[i];
        REAL sum_exp = (REAL)0;
        for (long i = 0; i < n; ++i) {
            const REAL e = ORA_EXP(row[i] - max_val);
            row[i] = e;
            sum_exp += e;
        }
        for (long i = 0; i < n; ++i) row[i] = row[i] / sum_exp;
        if (c->lse) c->lse[r] = (float)(max_val + ORA_LOG(sum_exp));
    }
}

static void FN(softmax_rows_inplace)(REAL* x, float* lse, long rows, long n) {
    FN(sm_ctx) c = {x, lse, n};
    ora_parallel_for(rows, FN(sm_task), &c);
}

/* ---- softmax backward (src/kernels/activations.rs:154-188):
 * dot = sum_i dy_i * y_i ; dx_i = y_i * (dy_i - dot). In place over dy. --- */
typedef struct {
    REAL* dy;
    const REAL* y;
    long n;
} FN(smb_ctx);

static void FN(smb_task)(void* vctx, long r0, long r1) {
    FN(smb_ctx)* c = (FN(smb_ctx)*)vctx;
    const long n = c->n;
    for (long r = r0; r < r1; ++r) {
        REAL* dy = c->dy + r * n;
        const REAL* y = c->y + r * n;
        REAL dot = (REAL)0;
        for (long i = 0; i < n; ++i) dot += dy[i] * y[i];
        for (long i = 0; i < n; ++i) dy[i] = y[i] * (dy[i] - dot);
    }
}

static void FN(softmax_backward_inplace)(REAL* dy, const REAL* y, long rows, long n) {
    FN(smb_ctx) c = {dy, y, n};
    ora_parallel_for(rows, FN(smb_task), &c);
}

static void FN(to_real)(const float* in, REAL* out, long n) {
    for (long i = 0; i < n; ++i) out[i] = (REAL)in[i];
}

static void FN(to_float)(const REAL* in, float* out, long n) {
    for (long i = 0; i < n; ++i) out[i] = (float)in[i];
}

/* scores = scale * (Q . K^T), then the causal mask (-inf above the
 * diagonal), then the row softmax in place. Follows
 * src/ops/flash_attention.rs:18-19: `q.batched_matmul(&k, true, scale)`
 * (src/tensor.rs:605-642: matmul, then `scalar_mul` by `scale`), then
 * `.softmax()`. The causal mask has no counterpart in the reference. */
static void FN(scores_softmax)(const REAL* q, const REAL* k, REAL* p, REAL* tmp, float* lse, long S,
                               long D, REAL scale, int causal) {
    FN(transpose)(k, tmp, S, D); /* K^T, D x S */
    FN(matmul)(q, tmp, p, S, D, S);
    FN(scale_inplace)(p, S * S, scale);
    if (causal) {
        for (long i = 0; i < S; ++i)
            for (long j = i + 1; j < S; ++j) p[i * S + j] = -(REAL)INFINITY;
    }
    FN(softmax_rows_inplace)(p, lse, S, S);
}

/* Attention forward over [BH, S, D] row-major slices.
 * O = softmax(scale * Q K^T [+ causal mask]) V, one (b,h) slice at a time,
 * as the reference's batched CPU fallback loops over the batch dimension
 * (src/tensor.rs:617-630). lse[BH*S] (may be NULL). */
int FN(ora_attn_fwd)(const float* q, const float* k, const float* v, float* o, float* lse, int BH,
                     int S, int D, float scale, int causal) {
    const long s = S, d = D;
    REAL* qs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* ks = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* vs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* os = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* p = (REAL*)malloc(sizeof(REAL) * s * s);
    REAL* tmp = (REAL*)malloc(sizeof(REAL) * s * (s > d ? s : d));
    if (!qs || !ks || !vs || !os || !p || !tmp) {
        free(qs); free(ks); free(vs); free(os); free(p); free(tmp);
        return -1;
    }
    for (long bh = 0; bh < BH; ++bh) {
        const long off = bh * s * d;
        FN(to_real)(q + off, qs, s * d);
        FN(to_real)(k + off, ks, s * d);
        FN(to_real)(v + off, vs, s * d);
        FN(scores_softmax)(qs, ks, p, tmp, lse ? lse + bh * s : NULL, s, d, (REAL)scale, causal);
        FN(matmul)(p, vs, os, s, s, d);
        FN(to_float)(os, o + off, s * d);
    }
    free(qs); free(ks); free(vs); free(os); free(p); free(tmp);
    return 0;
}

/* Attention backward, following src/ops/flash_attention.rs:16-39:
 *   P  = softmax(scale Q K^T)             (recomputed, :18-19)
 *   dV = P^T dO                           (:22)
 *   dP = dO V^T                           (:25)
 *   dS = softmax_backward(dP, P)          (:28, activations.rs:154-188)
 *   dQ = dS K   * scale                   (:31)
 *   dK = dS^T Q * scale                   (:34-36)
 * Every transpose is a true transpose. `ref_compat`=1 omits the two
 * `* scale` factors, reproducing the reference as written (it returns
 * dS K and dS^T Q, which are not the gradients of its own forward). */
int FN(ora_attn_bwd)(const float* q, const float* k, const float* v, const float* dout, float* dq,
                     float* dk, float* dv, int BH, int S, int D, float scale, int causal,
                     int ref_compat) {
    const long s = S, d = D;
    REAL* qs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* ks = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* vs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* dos = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* outs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* p = (REAL*)malloc(sizeof(REAL) * s * s);
    REAL* a = (REAL*)malloc(sizeof(REAL) * s * (s > d ? s : d));
    REAL* b = (REAL*)malloc(sizeof(REAL) * s * (s > d ? s : d));
    if (!qs || !ks || !vs || !dos || !outs || !p || !a || !b) {
        free(qs); free(ks); free(vs); free(dos); free(outs); free(p); free(a); free(b);
        return -1;
    }
    for (long bh = 0; bh < BH; ++bh) {
        const long off = bh * s * d;
        FN(to_real)(q + off, qs, s * d);
        FN(to_real)(k + off, ks, s * d);
        FN(to_real)(v + off, vs, s * d);
        FN(to_real)(dout + off, dos, s * d);
        FN(scores_softmax)(qs, ks, p, b, NULL, s, d, (REAL)scale, causal);
        /* dV = P^T dO */
        FN(transpose)(p, a, s, s);
        FN(matmul)(a, dos, outs, s, s, d);
        FN(to_float)(outs, dv + off, s * d);
        /* dP = dO V^T */
        FN(transpose)(vs, a, s, d); /* V^T, D x S */
        FN(matmul)(dos, a, b, s, d, s);
        /* dS = softmax_backward(dP, P), in place in b */
        FN(softmax_backward_inplace)(b, p, s, s);
        /* dQ = dS K (* scale) */
        FN(matmul)(b, ks, outs, s, s, d);
        if (!ref_compat) FN(scale_inplace)(outs, s * d, (REAL)scale);
        FN(to_float)(outs, dq + off, s * d);
        /* dK = dS^T Q (* scale) */
        FN(transpose)(b, a, s, s);
        FN(matmul)(a, qs, outs, s, s, d);
        if (!ref_compat) FN(scale_inplace)(outs, s * d, (REAL)scale);
        FN(to_float)(outs, dk + off, s * d);
    }
    free(qs); free(ks); free(vs); free(dos); free(outs); free(p); free(a); free(b);
    return 0;
}

/* Forward and backward together, over blocks of `rows` query rows, for
 * sequences whose S x S matrices do not fit in host memory (S = 32768 needs
 * 4 GiB per matrix). The formulas and the order of every sum are those of
 * ora_attn_fwd and ora_attn_bwd above (src/ops/flash_attention.rs:16-39),
 * so the results are the same bit for bit:
 *   * softmax and its backward are row-wise, so a block of rows sees exactly
 *     the rows of the full matrix;
 *   * under the causal mask the keys past the block's last row have P = 0
 *     and dS = 0 for every row of the block; they only add zeros to the
 *     full-matrix sums, so they are left out (keys [0, i1) for rows [i0, i1));
 *   * dK = dS^T Q and dV = P^T dO sum over query rows; the blocks are
 *     visited in order and each adds its rows in order (matmul_acc), which is
 *     the order of the full-matrix product; the scale is applied once at the
 *     end, as in ora_attn_bwd.
 * o, lse (may be NULL), dq, dk, dv: outputs, [BH, S, D] and [BH, S]. */
int FN(ora_attn_rows)(const float* q, const float* k, const float* v, const float* dout, float* o,
                      float* lse, float* dq, float* dk, float* dv, int BH, int S, int D, float scale,
                      int causal, int rows) {
    const long s = S, d = D;
    const long R = rows > 0 ? (rows < S ? rows : S) : S;
    REAL* qs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* ks = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* vs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* dos = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* dks = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* dvs = (REAL*)malloc(sizeof(REAL) * s * d);
    REAL* outs = (REAL*)malloc(sizeof(REAL) * R * d);
    REAL* tr = (REAL*)malloc(sizeof(REAL) * s * d);   /* K^T or V^T of the block's keys */
    REAL* p = (REAL*)malloc(sizeof(REAL) * R * s);    /* P of the block */
    REAL* dp = (REAL*)malloc(sizeof(REAL) * R * s);   /* dP, then dS */
    REAL* pt = (REAL*)malloc(sizeof(REAL) * R * s);   /* a transposed block */
    if (!qs || !ks || !vs || !dos || !dks || !dvs || !outs || !tr || !p || !dp || !pt) {
        free(qs); free(ks); free(vs); free(dos); free(dks); free(dvs); free(outs); free(tr);
        free(p); free(dp); free(pt);
        return -1;
    }
    for (long bh = 0; bh < BH; ++bh) {
        const long off = bh * s * d;
        FN(to_real)(q + off, qs, s * d);
        FN(to_real)(k + off, ks, s * d);
        FN(to_real)(v + off, vs, s * d);
        FN(to_real)(dout + off, dos, s * d);
        for (long i = 0; i < s * d; ++i) dks[i] = dvs[i] = (REAL)0;
        for (long i0 = 0; i0 < s; i0 += R) {
            const long i1 = (i0 + R) < s ? (i0 + R) : s;
            const long rb = i1 - i0;
            const long sk = causal ? i1 : s; /* keys that can be unmasked in this block */
            const REAL* qb = qs + i0 * d;
            const REAL* dob = dos + i0 * d;
            /* P = softmax(scale Q K^T [mask]) for rows [i0, i1) */
            FN(transpose)(ks, tr, sk, d);
            FN(matmul)(qb, tr, p, rb, d, sk);
            FN(scale_inplace)(p, rb * sk, (REAL)scale);
            if (causal) {
                for (long r = 0; r < rb; ++r)
                    for (long j = i0 + r + 1; j < sk; ++j) p[r * sk + j] = -(REAL)INFINITY;
            }
            FN(softmax_rows_inplace)(p, lse ? lse + bh * s + i0 : NULL, rb, sk);
            /* O = P V */
            FN(matmul)(p, vs, outs, rb, sk, d);
            FN(to_float)(outs, o + off + i0 * d, rb * d);
            /* dV += P^T dO */
            FN(transpose)(p, pt, rb, sk);
            FN(matmul_acc)(pt, dob, dvs, sk, rb, d);
            /* dP = dO V^T, then dS = softmax_backward(dP, P) */
            FN(transpose)(vs, tr, sk, d);
            FN(matmul)(dob, tr, dp, rb, d, sk);
            FN(softmax_backward_inplace)(dp, p, rb, sk);
            /* dQ = dS K * scale */
            FN(matmul)(dp, ks, outs, rb, sk, d);
            FN(scale_inplace)(outs, rb * d, (REAL)scale);
            FN(to_float)(outs, dq + off + i0 * d, rb * d);
            /* dK += dS^T Q */
            FN(transpose)(dp, pt, rb, sk);
            FN(matmul_acc)(pt, qb, dks, sk, rb, d);
        }
        FN(scale_inplace)(dks, s * d, (REAL)scale);
        FN(to_float)(dks, dk + off, s * d);
        FN(to_float)(dvs, dv + off, s * d);
    }
    free(qs); free(ks); free(vs); free(dos); free(dks); free(dvs); free(outs); free(tr);
    free(p); free(dp); free(pt);
    return 0;
}

#undef FN
#undef CAT
#undef CAT_
