// Host API of the SIMT / warp-MMA kernels: TACO codec, LayerNorm, GeLU backward,
// column sums, cross-entropy, grad norm + AdamW, embeddings, attention.
// All launches are asynchronous on `s`; return 0, a cudaError_t, or -1 for bad arguments.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace tn5b {
namespace kernels {
// TACO codec (taco.cu)
int taco_encode(const void* in, void* packet, int64_t elements, cudaStream_t s);
int taco_decode(const void* packet, void* out, int64_t elements, cudaStream_t s);
int taco_decode_reduce(const void* local, const void* packets, void* out, int64_t elements, int rank,
                       int world, cudaStream_t s);
int ordered_reduce(const void* local, const void* remote, void* out, int64_t elements, int rank,
                   int world, cudaStream_t s);
int diagnostic_delay(unsigned long long cycles, cudaStream_t s);
// LayerNorm / GeLU / column sums (norm.cu)
int layernorm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd,
                  int rows, int H, int64_t ld_x, int64_t ld_y, float eps, cudaStream_t s);
int layernorm_bwd_parts(int rows);
int layernorm_bwd(const void* dy, const void* x, const void* w, const float* mean, const float* rstd,
                  void* dx, void* dw, void* db, float* workspace, int rows, int H, const void* dres,
                  cudaStream_t s);
int column_sum(const void* g, int64_t ld, int rows, int cols, void* out, float* workspace,
               cudaStream_t s);
int gelu_bwd(const void* dy, const void* pre, void* dx, int64_t n, cudaStream_t s);
// Cross-entropy (loss.cu)
int ce_stats(const void* logits, int64_t ld, int M, int V, const int64_t* targets, int64_t start,
             float* rowmax, float* selected, cudaStream_t s);
int ce_sumexp(const void* logits, int64_t ld, int M, int V, const float* gmax, float* sumexp,
              cudaStream_t s);
int ce_loss(const float* gmax, const float* sumexp, const float* selected, int M, float* row_loss,
            float* mean_loss, float scale, cudaStream_t s);
int ce_bwd(void* logits, int64_t ld, int M, int V, const int64_t* targets, int64_t start,
           const float* gmax, const float* sumexp, float scale, const float* scale_ptr, cudaStream_t s);
// Optimizer (optim.cu)
int grad_sqsum_parts(int64_t n);
int grad_sqsum(const void* grad, int is_fp32, int64_t n, double* partial, double* out, int accumulate,
               cudaStream_t s);
int adamw_step(float* master, float* m, float* v, const void* grad, int grad_fp32, void* param,
               int64_t n, int64_t n_decay, const double* norm2, float max_norm, float lr, float wd,
               float beta1, float beta2, float eps, int step, int* status, cudaStream_t s);
// Embeddings (embed.cu)
int embed_fwd(const int64_t* tok, const void* E, void* out, int M, int H, int64_t start, int64_t V,
              cudaStream_t s);
int add_position(void* x, const void* P, int rows, int H, int64_t row0, int S, cudaStream_t s);
int position_bwd(const void* g, void* dP, int rows, int H, int64_t row0, int S, cudaStream_t s);
int64_t embed_bwd_workspace_ints(int M, int64_t V);
int embed_bwd(const int64_t* tok, const void* g, void* dE, int M, int H, int64_t start, int64_t V,
              int* workspace, int accumulate, cudaStream_t s);
// Attention (attention_tc.cu, attention_pre.cu)
// `trace` (optional, may be null): 16 progress words per CTA for stall diagnosis.
int attention_fwd_tc(const void* qkv, int64_t ld_qkv, void* out, int64_t ld_out, float* lse, int B, int S,
                     int H, float scale, int* status, uint64_t timeout_ns, cudaStream_t s,
                     unsigned long long* trace = nullptr);
int attention_bwd_pre(const void* out, int64_t ld_out, const void* dout, int64_t ld_dout, float* Dvec, int B,
                      int S, int H, cudaStream_t s);
int attention_bwd_tc(const void* qkv, int64_t ld_qkv, const void* dout, int64_t ld_dout, const float* lse,
                     const float* Dvec, void* dqkv, int64_t ld_dqkv, int B, int S, int H, float scale, int* status,
                     uint64_t timeout_ns, cudaStream_t s, unsigned long long* dbg_dkdv = nullptr,
                     unsigned long long* dbg_dq = nullptr);
}  // namespace kernels
}  // namespace tn5b
