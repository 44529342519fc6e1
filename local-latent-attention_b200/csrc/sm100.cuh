// Tensor-core (tcgen05 + TMA) kernels of the local branch for bf16
// activations on sm_100a. The SIMT kernels of local_simt.cu cover the rest.
#pragma once

#include "common.cuh"

namespace llattn {
namespace sm100 {

// True when the tcgen05 forward / backward kernels handle this geometry.
bool fwd_supported(const Geom& g, int elt_bytes);
bool bwd_supported(const Geom& g, int elt_bytes);

// Remote projection + gate + mix fused into the forward epilogue
// (models.py:392-438): remote_h = lat[t/qbs] W_rout[h]^T + b_rout[h] as one
// more tcgen05 MMA, then w = sigmoid(local.g_l + bias - remote.g_r) and
// mixed = w local + (1-w) remote per row. lat == nullptr: not fused (the
// caller runs the separate gate kernel). Needs latent_d_model == 64.
struct GateEpilogue {
  const void* lat;       // [B, Tq, 64] bf16
  const void* w_rout;    // [d, 64] bf16
  const float* b_rout;   // [d]
  const float* g_local;  // [hd]
  const float* g_remote; // [hd]
  void* mixed;           // [B, T, d] bf16
};
bool gate_fusable(const Geom& g);

cudaError_t launch_local_fwd(const Geom& g, const void* qkv, void* local_out, float* lse, const GateEpilogue& ep,
                             cudaStream_t s);
// dq into slot 0 of dqkv; dk, dv into slots 1 and 2. dl = gradient of the
// local output [B, T, H, hd] bf16; delta = rowsum(dl * local_out) [B, H, T].
cudaError_t launch_local_dq(const Geom& g, const void* qkv, const void* dl, const float* lse, const float* delta,
                            void* dqkv, cudaStream_t s);
cudaError_t launch_local_dkv(const Geom& g, const void* qkv, const void* dl, const float* lse,
                             const float* delta, void* dqkv, cudaStream_t s);

// Gate / r_out backward on tensor cores (needs gate_fusable): writes dl
// (bf16 [B,T,d]), delta [B,H,T], dr (bf16 [B,T,d]), dlat_tok (fp32 [B,T,64])
// and dg_part ([gate_bwd_ctas][gate_dg_floats]).
struct GateBwd {
  const void* local_out; const void* lat; const void* w_rout; const float* b_rout; const float* g_local;
  const float* g_remote; const void* dmixed; void* dl; float* delta; void* dr; float* dlat_tok; float* dg_part;
};
// Latent backward on tensor cores (latent head dim <= 64, at most 64 chunks,
// bf16): drq and per-split dgk/dgv partials [n_split][B][Nc][2][Ld] as the
// SIMT kernel writes them; n_split = latent_tc_splits(g) row splits.
bool latent_tc_ok(const Geom& g);
int latent_tc_splits(const Geom& g);
cudaError_t launch_latent_bwd_tc(const Geom& g, const void* rq, const void* gkv, const float* lat_lse,
                                 const float* dlat, void* drq, float* part, int n_split, cudaStream_t s);
// Latent backward on tensor cores for 64 < Nc <= 512 (bf16, latent head dim
// <= 64): a rows kernel (drq, and delta [B,Lh,Tq] fp32 into `delta`) then a
// keys kernel (dgk/dgv partials [n_split_keys][B][Nc][2][Ld] into `part`)
bool latent_tc_long_ok(const Geom& g);
cudaError_t launch_latent_bwd_tc_long(const Geom& g, const void* rq, const void* gkv, const float* lat_lse,
                                      const float* dlat, void* drq, float* delta, float* part, int n_split_keys,
                                      cudaStream_t s);
// Latent forward on tensor cores (bf16, latent head dim <= 64, up to 512
// chunks): lat [B,Tq,Ld], lat_lse [B,Lh,Tq]
bool latent_tc_fwd_ok(const Geom& g);
cudaError_t launch_latent_fwd_tc(const Geom& g, const void* rq, const void* gkv, void* lat, float* lat_lse,
                                 cudaStream_t s);
int gate_bwd_ctas(const Geom& g);
// floats per gate CTA in dg_part: dg_local [hd], then per head S1_h [64] =
// sum_t ds lat[t] and S0_h = sum_t ds, from which dg_remote follows linearly
int gate_dg_floats(const Geom& g);
// dg_remote [hd] from the CTA-summed dg partials (dg_sum [gate_dg_floats])
cudaError_t launch_gate_dgr_finalize(const Geom& g, const float* dg_sum, const void* w_rout, const float* b_rout,
                                     float* dg_remote, cudaStream_t s);
cudaError_t launch_gate_bwd(const Geom& g, const GateBwd& a, cudaStream_t s);
// dW_rout / db_rout partials over n_split token ranges: dw_part [n_split][d*64],
// db_part [n_split][d]; dr bf16 [B*T, d] (d a multiple of 64), lat [B,Tq,64].
cudaError_t launch_rout_dw(const Geom& g, const void* dr, const void* lat, float* dw_part, float* db_part,
                           int n_split, cudaStream_t s);
cudaError_t launch_dlat_rowsum(const Geom& g, const float* dlat_tok, float* dlat, cudaStream_t s);

// C[M, N] = A[M, K] B[N, K]^T on the tensor cores (bf16 operands, fp32
// accumulation); a_mn / b_mn: operand stored [K, M] / [K, N] (MN-major)
// instead of [M, K] / [N, K]; lda / ldb: row strides in elements (multiples
// of 8). Output row m goes to row (m / rows_per_group) * group_stride +
// (m % rows_per_group) * row_step of C (rows_per_group 0: plain rows). K is
// split over `splits` CTAs along z, split z writing C + z * split_stride;
// colsum (optional, fp32 [splits][M] at colsum_split apart) = sum_k A[m, k].
struct GemmOut {
  void* C;
  int64_t ldc;
  int out_bf16;
  int64_t split_stride;
  const float* bias;
  int rows_per_group, group_stride, row_step;
  float* colsum;
  int64_t colsum_split;
};
cudaError_t launch_gemm(const Geom& g, int M, int N, int K, const void* A, int64_t lda, int a_mn, const void* B,
                        int64_t ldb, int b_mn, const GemmOut& o, int splits, cudaStream_t s);

// Reads (and optionally clears) the device fault word of the current device:
// bits set by a tensor-core kernel whose bounded wait ran out.
unsigned read_fault_word(bool reset);

}  // namespace sm100
}  // namespace llattn
