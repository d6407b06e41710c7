// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/haelixe_cuda.h"

namespace hx {

// Device status word written by kernels whose bounded waits expire.
// 0 = fine; otherwise a code naming the wait that gave up.
struct DeviceStatus {
    int code;
    int where;
    int block;
    int pad;
};

struct RopeTable {
    int S, D;
    uint32_t base_bits;
    float2* tab;  // device, [S][D/2]
};

struct Arena {
    cudaMemPool_t pool = nullptr;
    std::mutex mu;
    std::unordered_map<uint64_t, std::vector<void*>> free_list;  // bin -> slabs
    std::unordered_map<void*, uint64_t> live;                    // slab -> bin
    uint64_t live_bytes = 0, cached_bytes = 0, hits = 0, misses = 0;
    uint64_t limit = 0;  // bytes the arena may hold (live + parked); 0 = no limit
};

}  // namespace hx

struct hx_ctx {
    int device = 0;
    int sm_count = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    hx::Arena arena;
    hx::DeviceStatus* status = nullptr;  // device memory
    int last_path = 0;
    uint64_t kernel_launches = 0;
    int force_simt = 0;
    mutable std::mutex err_mu;
    std::string last_error;
    std::mutex rope_mu;
    std::vector<hx::RopeTable> rope_tables;  // (cos, sin) tables, freed with the context
    std::mutex blas_mu;
    void* blas = nullptr;  // cublasHandle_t for the f32 Linear GEMMs, created on first use
    // bf16 Linear GEMMs: 0 = tcgen05 kernel where it applies (tile from the
    // shape), 1 = cuBLAS, 2/3/4 = tcgen05 with tiles 128x128 / 128x256 / 256x256
    int gemm_backend = 0;
    int last_gemm_path = 0;  // 1 cuBLAS, 2 tcgen05 (the last Linear GEMM of this context)
};

namespace hx {

// Per-operand view: element strides, D contiguous.
struct AttnDims {
    int B, H, S, D;
    int64_t sb, sh, ss;
};

inline AttnDims dims_of(const hx_attn_shape& s) {
    return AttnDims{s.B, s.H, s.S, s.D, s.stride_b, s.stride_h, s.stride_s};
}

int set_error(const hx_ctx* ctx, int status, const char* fmt, ...);
int check_cuda(const hx_ctx* ctx, cudaError_t e, const char* what);

// ---- SIMT kernels (attn_simt.cu): any head_dim <= 256, f32 or bf16 ----
cudaError_t simt_attn_fwd(cudaStream_t st, hx_dtype dt, const AttnDims& d, const void* q,
                          const void* k, const void* v, void* o, float* lse, float scale,
                          int causal);
cudaError_t simt_attn_bwd(cudaStream_t st, hx_dtype dt, const AttnDims& d, const void* q,
                          const void* k, const void* v, const void* o, const void* dout,
                          const float* lse, void* dq, void* dk, void* dv, float* delta,
                          float scale, int causal);

// ---- tcgen05 kernels (attn_fwd_sm100.cu / attn_bwd_sm100.cu): bf16, D in {64,128} ----
bool sm100_supported(hx_dtype dt, const AttnDims& d);
cudaError_t sm100_attn_fwd(cudaStream_t st, int sm_count, DeviceStatus* status,
                           const AttnDims& d, const void* q, const void* k, const void* v,
                           void* o, float* lse, float scale, int causal);
bool sm100_bwd_supported(hx_dtype dt, const AttnDims& d);
uint64_t sm100_bwd_workspace_bytes(const AttnDims& d);
cudaError_t sm100_attn_bwd(cudaStream_t st, int sm_count, DeviceStatus* status,
                           const AttnDims& d, const void* q, const void* k, const void* v,
                           const void* o, const void* dout, const float* lse, void* dq,
                           void* dk, void* dv, void* workspace, float scale, int causal,
                           const float2* rope_tab = nullptr);

// ---- tcgen05 kernels for f32 I/O by operand splitting (attn_split_sm100.cu): D in {64,128} ----
// Each f32 operand as bf16 hi + lo planes, every product as three bf16 UMMAs.
bool split_supported(hx_dtype dt, const AttnDims& d);
uint64_t split_fwd_workspace_bytes(const AttnDims& d);
uint64_t split_bwd_workspace_bytes(const AttnDims& d);
cudaError_t split_attn_fwd(cudaStream_t st, int sm_count, DeviceStatus* status, const AttnDims& d, const void* q,
                           const void* k, const void* v, void* o, float* lse, float scale, int causal, void* ws);
// dq/dk/dv are f32; dq is zeroed and accumulated in place (red.global.add).
cudaError_t split_attn_bwd(cudaStream_t st, int sm_count, DeviceStatus* status, const AttnDims& d, const void* q,
                           const void* k, const void* v, const void* o, const void* dout, const float* lse,
                           void* dq, void* dk, void* dv, void* ws, float scale, int causal);

// ---- the attention block around the kernel (mha_ops.cu) ----
cudaError_t rmsnorm_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* x, const void* w, void* y,
                        int rows, int hidden, float eps);
cudaError_t rmsnorm_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* g, const void* x, const void* w,
                        void* dx, float* dw, float* scratch, int rows, int hidden, float eps);
cudaError_t rows_init(cudaStream_t st, int sm_count, hx_dtype dt, void* y, const void* res, const void* b,
                      int64_t rows, int cols);
cudaError_t cross_entropy(cudaStream_t st, hx_dtype dt, const void* logits, const uint32_t* targets,
                          float* row_loss, float* loss, void* dlogits, int rows, int classes);
cudaError_t adamw_step(cudaStream_t st, int sm_count, const hx_adamw_tensor* tensors, int count, float lr,
                       float beta1, float beta2, float eps, float weight_decay, float bc1, float bc2);
cudaError_t embedding_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* table, const uint32_t* ids,
                          void* out, int64_t tokens, int vocab, int dim);
cudaError_t embedding_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* dout, const uint32_t* ids,
                          float* dtable, int64_t tokens, int vocab, int dim);
cudaError_t gelu_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* x, void* y, int64_t n);
cudaError_t add(cudaStream_t st, int sm_count, hx_dtype dt, const void* a, const void* b, void* out, int64_t n);
cudaError_t gelu_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* g, const void* x, void* dx, int64_t n);
// db[c] = sum over rows of dy[r, c]; scratch holds col_scratch_floats(rows, cols) floats.
cudaError_t col_sum(cudaStream_t st, hx_dtype dt, const void* dy, void* db, float* scratch, int64_t rows, int cols);
int64_t col_scratch_floats(int64_t rows, int cols);
int64_t rmsnorm_bwd_scratch_floats(int64_t rows, int hidden);

// ---- failure-path self-test (selftest.cu) ----
cudaError_t selftest_wait_timeout(cudaStream_t st, DeviceStatus* status);

// ---- tcgen05 GEMM (gemm_sm100.cu): row-major bf16, f32 accumulation ----
// C[M,N] = A'[M,K] B'[K,N] (+ bias[N]) (+ R[M,N]); A' = A (K-major) or A^T
// (a_mn), B' = B (b_mn, N contiguous) or B^T (K-major). cudaErrorNotSupported
// when the operands do not meet TMA's layout rules (the caller uses cuBLAS).
bool gemm_bf16_supported(bool a_mn, bool b_mn, int M, int N, int K, const void* A, int64_t lda, const void* B,
                         int64_t ldb, const void* C, int64_t ldc, const void* R, int64_t ldr, const void* bias);
// tile: 0 = chosen from the shape, 1 = 128 x 128, 2 = 128 x 256, 3 = 256 x 256.
cudaError_t gemm_bf16(cudaStream_t st, int sm_count, DeviceStatus* status, bool a_mn, bool b_mn, int M, int N,
                      int K, const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                      const void* R, int64_t ldr, const void* bias, int tile = 0);

// ---- head reassembly (heads.cu) ----
cudaError_t reassemble_heads(cudaStream_t st, int elem_bytes, const void* src, void* dst, int n,
                             int B, int Hs, int S, int D, int layout, int sm_count);

// Counts kernel launches of the calling thread; hx_api attributes them to a context.
void note_launch();
uint64_t launches_of_this_thread();

// ---- RoPE (rope.cu) ----
// Fills tab[S][D/2] with (cos, sin) of s * inv_freq[i].
cudaError_t rope_table(cudaStream_t st, int S, int D, const float* inv_freq_host, float2* tab);
// With x2/out2: a second tensor of the same shape and strides in the same launch.
cudaError_t rope_apply(cudaStream_t st, int sm_count, hx_dtype dt, const AttnDims& d,
                       const void* x, void* out, const float2* tab, float sign, const void* x2 = nullptr,
                       void* out2 = nullptr);

}  // namespace hx
