// Shared device helpers of libllattn: geometry, masks, dtype conversion.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "llattn.h"

namespace llattn {

using bf16 = __nv_bfloat16;

// Geometry of one call, derived once on the host (see api.cu: make_geom).
// Every size the kernels need, in the reference's terms:
//   d = H*hd, Ld = Lh*ldh, bsL = local query-block span (models.py:249),
//   cs/Nc = latent chunk size/count (models.py:175-183),
//   qbs/Tq = latent query block size/row count (models.py:216-219; 1/T when
//   queries are token-wise).
struct Geom {
  int B, T, H, hd, d, Lh, ldh, Ld;
  int W, bsL, cs, Nc, qbs, Tq;
  // sequence shards: row 0 of this call is global position `off` of a
  // sequence of `T_total` tokens; bsL, cs, Nc and qbs follow T_total, the
  // masks and chunk ids follow global positions (off = 0, T_total = T for
  // a whole sequence)
  int off, T_total;
  // row strides (elements) of qkv (read) and dqkv (written): 3d unless the
  // rows sit in a wider buffer
  int ldq, ldd;
  float gate_bias;
  float scale;      // 1/sqrt(hd)
  float lat_scale;  // 1/sqrt(ldh)
  // host-mapped fault word (pinned, zero-copy): set by a kernel that gave up
  // on a bounded wait; nullptr disables the mirror
  volatile unsigned* fault_host;
};

__host__ __device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes) only when
// this (kernel, device) has not been given at least `bytes` yet: the
// attribute is per-device state of the function, so the call (a driver
// round trip) is made once per kernel instance and device instead of on
// every launch. Thread-safe (api.cu).
cudaError_t set_smem_attr(const void* kernel, int bytes);
template <typename K>
cudaError_t set_smem_once(K kernel, int bytes) {
  return set_smem_attr(reinterpret_cast<const void*>(kernel), bytes);
}

// First key visible from query t (inclusive); the last is t-1. Mask of
// models.py:245-292: 0 < t-j <= W and j >= max(0, qs(t)-W+1), where qs(t) is
// the first row of t's bsL-block.
__host__ __device__ __forceinline__ int local_lo(const Geom& g, int t) {
  const int tg = t + g.off;  // global position
  int qs = (tg / g.bsL) * g.bsL;
  int lo = tg - g.W;
  int lo2 = qs - g.W + 1;
  lo = lo > lo2 ? lo : lo2;
  lo = (lo > 0 ? lo : 0) - g.off;  // back to this call's rows (a shard holds the keys it needs)
  return lo > 0 ? lo : 0;
}

// Last query (inclusive, this call's rows) that sees key j: t - j <= W and t
// before the end of the bsL-block holding global position j + W - 1.
__host__ __device__ __forceinline__ int local_hi(const Geom& g, int j) {
  const int jg = j + g.off;
  const int a = jg + g.W, bnd = ((jg + g.W - 1) / g.bsL + 1) * g.bsL - 1;
  const int hi = (a < bnd ? a : bnd) - g.off;
  return hi < g.T - 1 ? hi : g.T - 1;
}

__host__ __device__ __forceinline__ bool local_visible(const Geom& g, int t, int j) {
  return j < t && j >= local_lo(g, t);
}

// Latent chunk count visible from latent query row r (chunks j < qid(r)),
// models.py:208-212, 227-229, 363-365.
__host__ __device__ __forceinline__ int row_qid(const Geom& g, int r) {
  int t = g.off + r * g.qbs;
  int c = t / g.cs;
  return c < g.Nc - 1 ? c : g.Nc - 1;
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return to_f<T>(*p); }
template <typename T>
__device__ __forceinline__ void stf(T* p, float v) { *p = from_f<T>(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Launch helpers implemented per .cu file; all return cudaError_t of the
// launch so api.cu can turn it into a status.
template <typename T>
cudaError_t launch_pool_fwd(const Geom& g, int mode, const T* x, T* out, int64_t d, cudaStream_t s);
template <typename T>
cudaError_t launch_pool_bwd(const Geom& g, int mode, const T* dout, T* dx, int64_t d, int accumulate,
                            cudaStream_t s);
template <typename T>
cudaError_t launch_pool_proj_fwd(const Geom& g, const T* z, int64_t ldz, const T* b_rkv, const T* b_rq, T* gkv,
                                 T* rq, cudaStream_t s);
template <typename T>
cudaError_t launch_pool_proj_bwd(const Geom& g, const T* dgkv, const T* drq, T* dz, int64_t ldz, cudaStream_t s);
// out[c] = sum_r g[r, c] over a row-major [rows, cols] matrix; part holds
// colsum_splits(rows, cols, sizeof(T)) x cols floats
int colsum_splits(int64_t rows, int64_t cols, int elem_bytes);
int sm_count();  // SMs of the current device
template <typename T, typename To = T>
cudaError_t launch_colsum(const T* g, int64_t rows, int64_t cols, float* part, To* out, cudaStream_t s,
                          int64_t ld = 0);  // ld: row stride in elements (0 = cols)
template <typename To>
cudaError_t launch_reduce_parts(const float* part, int n_part, int64_t n, To* out, cudaStream_t s);

template <typename T>
cudaError_t launch_latent_fwd(const Geom& g, const T* rq, const T* gkv, T* lat, float* lat_lse,
                              cudaStream_t s);
// Latent backward: drq and per-CTA partials of dgk/dgv ([n_split * n_kg][B][Nc][2][Ld],
// every entry written). n_kg > 1 (more than one 64-key tile) splits the key
// tiles of each row split over n_kg CTAs; their drq goes through drq_part
// ([n_kg][B][Tq][Ld] fp32) and a fixed-order sum.
template <typename T>
cudaError_t launch_latent_bwd(const Geom& g, const T* rq, const T* gkv, const float* lat_lse,
                              const float* dlat, T* drq, float* dgkv_part, int n_split, int n_kg, float* drq_part,
                              cudaStream_t s);
// One decode step (decode.cu): qkv cache [B, cache_len, 3, H, hd] with rows
// 0..T-1 filled, rq_row [B, Ld], gkv [B, Nc, 2, Ld] -> out [B, d] (row T-1).
template <typename T>
cudaError_t launch_decode(const Geom& g, int64_t cache_len, const T* qkv, const T* rq_row, const T* gkv,
                          const T* w_rout, const float* b_rout, const float* g_local, const float* g_remote, T* out,
                          cudaStream_t s);
template <typename T>
cudaError_t launch_latent_reduce(const Geom& g, const float* dgkv_part, int n_split, T* dgkv,
                                 cudaStream_t s);

template <typename T>
cudaError_t launch_local_fwd_simt(const Geom& g, const T* qkv, T* local_out, float* lse,
                                  cudaStream_t s);
template <typename T>
cudaError_t launch_local_bwd_simt(const Geom& g, const T* qkv, const T* dl, const float* lse,
                                  const float* delta, T* dqkv, cudaStream_t s);

template <typename T>
cudaError_t launch_gate_fwd(const Geom& g, const T* local_out, const T* lat, const T* w_rout,
                            const float* b_rout, const float* g_local, const float* g_remote,
                            T* mixed, cudaStream_t s);
template <typename T>
cudaError_t launch_gate_bwd(const Geom& g, const T* local_out, const T* lat, const T* w_rout,
                            const float* b_rout, const float* g_local, const float* g_remote,
                            const T* dmixed, T* dl, float* delta, float* drow, float* dg_part,
                            int tok_per_cta, cudaStream_t s);
template <typename T>
cudaError_t launch_rout_bwd(const Geom& g, const float* drow, const T* lat, const T* w_rout,
                            float* dlat, float* dw_part, int n_split, cudaStream_t s);
// Gate and mix with the remote projection precomputed (bf16; see gate.cu):
// forward in place over `mixed`, which holds the remote rows on entry (token
// t's at row t, query block r's at row r * qbs); backward with the remote
// rows rem [B*Tq, d], writing dl, delta, dr (per token, or per query block
// summed over its tokens) and gate_rmem_ctas(g) partials [2 hd] of dg.
int gate_rmem_ctas(const Geom& g);
cudaError_t launch_gate_mix_rmem(const Geom& g, const bf16* local_out, const float* g_local, const float* g_remote,
                                 bf16* mixed, cudaStream_t s);
cudaError_t launch_gate_bwd_rmem(const Geom& g, const bf16* local_out, const bf16* rem, const float* g_local,
                                 const float* g_remote, const bf16* dmixed, bf16* dl, float* delta, bf16* dr,
                                 float* dg_part, cudaStream_t s);
cudaError_t launch_reduce_rows(const float* part, int n_part, int64_t n, float* out,
                               cudaStream_t s);

}  // namespace llattn
