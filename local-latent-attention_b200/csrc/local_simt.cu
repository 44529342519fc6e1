// Local branch, exact fp32 path: windowed causal attention with the
// reference's blockwise mask (models.py:232-305), forward and backward, on
// fp32 FMAs. This is the path of fp32 activations (the 1e-4 parity config)
// and of head dims the tensor-core kernels do not cover.
//
// q/k/v are read in place from the qkv projection output [B, T, 3, H, hd]
// (row stride 3*H*hd); dq/dk/dv are written into the same layout, so the
// qkv projection's backward consumes them without a copy.
//
// Tiles: 32 query rows x 32 keys per step, 128 threads; thread (i = tid/4,
// c = tid%4) owns query row i, keys c+4u and head-dim columns c+4m. Shared
// rows are padded by one float so the 8 rows a warp touches hit 8 banks.
#include <math.h>

#include "common.cuh"

namespace llattn {
namespace {

constexpr int QT = 32;
constexpr int KT = 32;
constexpr int NT = 128;

template <typename T, int HD>
__device__ __forceinline__ void load_rows(float (*dst)[HD + 1], const T* base, int64_t row_stride,
                                          int t0, int n_rows, int t_lim, int hd, float mul) {
  for (int idx = threadIdx.x; idx < n_rows * HD; idx += NT) {
    const int r = idx / HD, e = idx % HD, t = t0 + r;
    dst[r][e] = (t >= 0 && t < t_lim && e < hd) ? to_f<T>(base[(int64_t)t * row_stride + e]) * mul : 0.f;
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(NT) local_fwd_simt_kernel(Geom g, const T* __restrict__ qkv,
                                                            T* __restrict__ local_out,
                                                            float* __restrict__ lse) {
  extern __shared__ float smem_lf[];
  float(*sq)[HD + 1] = reinterpret_cast<float(*)[HD + 1]>(smem_lf);
  float(*sk)[HD + 1] = sq + QT;
  float(*sv)[HD + 1] = sk + KT;
  float(*sp)[KT + 1] = reinterpret_cast<float(*)[KT + 1]>(sv + KT);
  const int q0 = blockIdx.x * QT, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, i = tid / 4, c = tid % 4;
  const int64_t rs = g.ldq;  // qkv row stride
  const T* qb = qkv + (int64_t)b * g.T * rs + (int64_t)h * g.hd;
  load_rows<T, HD>(sq, qb, rs, q0, QT, g.T, g.hd, g.scale);

  const int t = q0 + i;
  const int qlast = min(q0 + QT, g.T) - 1;
  const int klo = local_lo(g, q0), khi = qlast - 1;
  const int my_lo = t < g.T ? local_lo(g, t) : 0;
  float m = -INFINITY, l = 0.f;
  float o[HD / 4];
#pragma unroll
  for (int u = 0; u < HD / 4; ++u) o[u] = 0.f;

  for (int k0 = klo; k0 <= khi; k0 += KT) {
    __syncthreads();
    load_rows<T, HD>(sk, qb + g.d, rs, k0, KT, khi + 1, g.hd, 1.f);
    load_rows<T, HD>(sv, qb + 2 * g.d, rs, k0, KT, khi + 1, g.hd, 1.f);
    __syncthreads();
    float s[KT / 4];
    float mx = -INFINITY;
#pragma unroll
    for (int u = 0; u < KT / 4; ++u) {
      const int jj = c + 4 * u, j = k0 + jj;
      float dot = 0.f;
#pragma unroll 16
      for (int e = 0; e < HD; ++e) dot = fmaf(sq[i][e], sk[jj][e], dot);
      const bool vis = t < g.T && j <= khi && j < t && j >= my_lo;
      s[u] = vis ? dot : -INFINITY;
      mx = fmaxf(mx, s[u]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m, mx);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = expf(m - m_use);
    float psum = 0.f;
#pragma unroll
    for (int u = 0; u < KT / 4; ++u) {
      const float p = expf(s[u] - m_use);
      sp[i][c + 4 * u] = p;
      psum += p;
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    l = l * alpha + psum;
    m = m_new;
#pragma unroll
    for (int u = 0; u < HD / 4; ++u) o[u] *= alpha;
    __syncthreads();
    for (int jj = 0; jj < KT; ++jj) {
      const float p = sp[i][jj];
#pragma unroll
      for (int u = 0; u < HD / 4; ++u) o[u] = fmaf(p, sv[jj][c + 4 * u], o[u]);
    }
  }
  if (t < g.T) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T* dst = local_out + ((int64_t)b * g.T + t) * g.d + (int64_t)h * g.hd;
#pragma unroll
    for (int u = 0; u < HD / 4; ++u) {
      const int e = c + 4 * u;
      if (e < g.hd) dst[e] = from_f<T>(o[u] * inv);
    }
    if (c == 0) lse[((int64_t)b * g.H + h) * g.T + t] = l > 0.f ? m + logf(l) : INFINITY;
  }
}

// dQ = scale * sum_j dS_ij k_j with dS = P (dP - D), P = exp(s - lse),
// dP = dO . v_j. One CTA per 32 query rows.
template <typename T, int HD>
__global__ void __launch_bounds__(NT) local_dq_simt_kernel(Geom g, const T* __restrict__ qkv,
                                                           const T* __restrict__ dl,
                                                           const float* __restrict__ lse,
                                                           const float* __restrict__ delta,
                                                           T* __restrict__ dqkv) {
  extern __shared__ float smem_dq[];
  float(*sq)[HD + 1] = reinterpret_cast<float(*)[HD + 1]>(smem_dq);
  float(*sdo)[HD + 1] = sq + QT;
  float(*sk)[HD + 1] = sdo + QT;
  float(*sv)[HD + 1] = sk + KT;
  float(*sds)[KT + 1] = reinterpret_cast<float(*)[KT + 1]>(sv + KT);
  const int q0 = blockIdx.x * QT, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, i = tid / 4, c = tid % 4;
  const int64_t rs = g.ldq;  // qkv row stride
  const T* qb = qkv + (int64_t)b * g.T * rs + (int64_t)h * g.hd;
  load_rows<T, HD>(sq, qb, rs, q0, QT, g.T, g.hd, g.scale);
  load_rows<T, HD>(sdo, dl + (int64_t)b * g.T * g.d + (int64_t)h * g.hd, g.d, q0, QT, g.T, g.hd, 1.f);

  const int t = q0 + i;
  const int qlast = min(q0 + QT, g.T) - 1;
  const int klo = local_lo(g, q0), khi = qlast - 1;
  const int my_lo = t < g.T ? local_lo(g, t) : 0;
  const float my_lse = t < g.T ? lse[((int64_t)b * g.H + h) * g.T + t] : INFINITY;
  const float my_d = t < g.T ? delta[((int64_t)b * g.H + h) * g.T + t] : 0.f;
  float acc[HD / 4];
#pragma unroll
  for (int u = 0; u < HD / 4; ++u) acc[u] = 0.f;

  for (int k0 = klo; k0 <= khi; k0 += KT) {
    __syncthreads();
    load_rows<T, HD>(sk, qb + g.d, rs, k0, KT, khi + 1, g.hd, 1.f);
    load_rows<T, HD>(sv, qb + 2 * g.d, rs, k0, KT, khi + 1, g.hd, 1.f);
    __syncthreads();
#pragma unroll
    for (int u = 0; u < KT / 4; ++u) {
      const int jj = c + 4 * u, j = k0 + jj;
      float sdot = 0.f, pdot = 0.f;
#pragma unroll 16
      for (int e = 0; e < HD; ++e) {
        sdot = fmaf(sq[i][e], sk[jj][e], sdot);
        pdot = fmaf(sdo[i][e], sv[jj][e], pdot);
      }
      const bool vis = t < g.T && j <= khi && j < t && j >= my_lo;
      const float p = vis ? expf(sdot - my_lse) : 0.f;
      sds[i][jj] = p * (pdot - my_d);
    }
    __syncthreads();
    for (int jj = 0; jj < KT; ++jj) {
      const float ds = sds[i][jj];
#pragma unroll
      for (int u = 0; u < HD / 4; ++u) acc[u] = fmaf(ds, sk[jj][c + 4 * u], acc[u]);
    }
  }
  if (t < g.T) {
    T* dst = dqkv + ((int64_t)b * g.T + t) * g.ldd + (int64_t)h * g.hd;
#pragma unroll
    for (int u = 0; u < HD / 4; ++u) {
      const int e = c + 4 * u;
      if (e < g.hd) dst[e] = from_f<T>(acc[u] * g.scale);
    }
  }
}

// dV_j = sum_i P_ij dO_i, dK_j = scale * sum_i dS_ij q_i. One CTA per 32 keys,
// looping over the queries that can see them: t in [j0+1, j0+31+W].
template <typename T, int HD>
__global__ void __launch_bounds__(NT) local_dkv_simt_kernel(Geom g, const T* __restrict__ qkv,
                                                            const T* __restrict__ dl,
                                                            const float* __restrict__ lse,
                                                            const float* __restrict__ delta,
                                                            T* __restrict__ dqkv) {
  extern __shared__ float smem_dkv[];
  float(*sk)[HD + 1] = reinterpret_cast<float(*)[HD + 1]>(smem_dkv);
  float(*sv)[HD + 1] = sk + KT;
  float(*sq)[HD + 1] = sv + KT;
  float(*sdo)[HD + 1] = sq + QT;
  float(*sp)[QT + 1] = reinterpret_cast<float(*)[QT + 1]>(sdo + QT);
  float(*sds)[QT + 1] = sp + KT;
  float* slse = reinterpret_cast<float*>(sds + KT);
  float* sd = slse + QT;
  int* slo = reinterpret_cast<int*>(sd + QT);
  const int j0 = blockIdx.x * KT, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, jr = tid / 4, c = tid % 4;
  const int64_t rs = g.ldq;  // qkv row stride
  const T* qb = qkv + (int64_t)b * g.T * rs + (int64_t)h * g.hd;
  const T* db = dl + (int64_t)b * g.T * g.d + (int64_t)h * g.hd;
  const float* lse_b = lse + ((int64_t)b * g.H + h) * g.T;
  const float* d_b = delta + ((int64_t)b * g.H + h) * g.T;
  load_rows<T, HD>(sk, qb + g.d, rs, j0, KT, g.T, g.hd, 1.f);
  load_rows<T, HD>(sv, qb + 2 * g.d, rs, j0, KT, g.T, g.hd, 1.f);
  const int j = j0 + jr;
  float adk[HD / 4], adv[HD / 4];
#pragma unroll
  for (int u = 0; u < HD / 4; ++u) adk[u] = adv[u] = 0.f;
  const int t_end = min(g.T - 1, j0 + KT - 1 + g.W);  // inclusive

  for (int t0 = j0 + 1; t0 <= t_end; t0 += QT) {
    __syncthreads();
    load_rows<T, HD>(sq, qb, rs, t0, QT, t_end + 1, g.hd, 1.f);
    load_rows<T, HD>(sdo, db, g.d, t0, QT, t_end + 1, g.hd, 1.f);
    if (tid < QT) {
      const int t = t0 + tid;
      const bool ok = t <= t_end;
      slse[tid] = ok ? lse_b[t] : INFINITY;
      sd[tid] = ok ? d_b[t] : 0.f;
      slo[tid] = ok ? local_lo(g, t) : 0x7fffffff;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < QT / 4; ++u) {
      const int ii = c + 4 * u, t = t0 + ii;
      float sdot = 0.f, pdot = 0.f;
#pragma unroll 16
      for (int e = 0; e < HD; ++e) {
        sdot = fmaf(sk[jr][e], sq[ii][e], sdot);
        pdot = fmaf(sv[jr][e], sdo[ii][e], pdot);
      }
      const bool vis = j < g.T && t <= t_end && j < t && j >= slo[ii];
      const float p = vis ? expf(sdot * g.scale - slse[ii]) : 0.f;
      sp[jr][ii] = p;
      sds[jr][ii] = p * (pdot - sd[ii]);
    }
    __syncthreads();
    for (int ii = 0; ii < QT; ++ii) {
      const float p = sp[jr][ii], ds = sds[jr][ii];
#pragma unroll
      for (int u = 0; u < HD / 4; ++u) {
        adv[u] = fmaf(p, sdo[ii][c + 4 * u], adv[u]);
        adk[u] = fmaf(ds, sq[ii][c + 4 * u], adk[u]);
      }
    }
  }
  if (j < g.T) {
    T* dst = dqkv + ((int64_t)b * g.T + j) * g.ldd + (int64_t)h * g.hd;
#pragma unroll
    for (int u = 0; u < HD / 4; ++u) {
      const int e = c + 4 * u;
      if (e < g.hd) {
        dst[g.d + e] = from_f<T>(adk[u] * g.scale);
        dst[2 * g.d + e] = from_f<T>(adv[u]);
      }
    }
  }
}

template <typename T, int HD>
cudaError_t fwd_hd(const Geom& g, const T* qkv, T* out, float* lse, cudaStream_t s) {
  const size_t sm = sizeof(float) * ((QT + 2 * KT) * (HD + 1) + QT * (KT + 1));
  cudaError_t e = set_smem_once(local_fwd_simt_kernel<T, HD>, (int)sm);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, QT), g.H, g.B);
  local_fwd_simt_kernel<T, HD><<<grid, NT, sm, s>>>(g, qkv, out, lse);
  return cudaGetLastError();
}

template <typename T, int HD>
cudaError_t bwd_hd(const Geom& g, const T* qkv, const T* dl, const float* lse, const float* delta,
                   T* dqkv, cudaStream_t s) {
  const size_t sm1 = sizeof(float) * ((2 * QT + 2 * KT) * (HD + 1) + QT * (KT + 1));
  const size_t sm2 = sizeof(float) * ((2 * QT + 2 * KT) * (HD + 1) + 2 * KT * (QT + 1) + 3 * QT);
  cudaError_t e = set_smem_once(local_dq_simt_kernel<T, HD>, (int)sm1);
  if (e != cudaSuccess) return e;
  e = set_smem_once(local_dkv_simt_kernel<T, HD>, (int)sm2);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, QT), g.H, g.B);
  local_dq_simt_kernel<T, HD><<<grid, NT, sm1, s>>>(g, qkv, dl, lse, delta, dqkv);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  dim3 grid2(cdiv(g.T, KT), g.H, g.B);
  local_dkv_simt_kernel<T, HD><<<grid2, NT, sm2, s>>>(g, qkv, dl, lse, delta, dqkv);
  return cudaGetLastError();
}

}  // namespace

template <typename T>
cudaError_t launch_local_fwd_simt(const Geom& g, const T* qkv, T* local_out, float* lse, cudaStream_t s) {
  if (g.hd <= 32) return fwd_hd<T, 32>(g, qkv, local_out, lse, s);
  if (g.hd <= 64) return fwd_hd<T, 64>(g, qkv, local_out, lse, s);
  return fwd_hd<T, 128>(g, qkv, local_out, lse, s);
}

template <typename T>
cudaError_t launch_local_bwd_simt(const Geom& g, const T* qkv, const T* dl, const float* lse,
                                  const float* delta, T* dqkv, cudaStream_t s) {
  if (g.hd <= 32) return bwd_hd<T, 32>(g, qkv, dl, lse, delta, dqkv, s);
  if (g.hd <= 64) return bwd_hd<T, 64>(g, qkv, dl, lse, delta, dqkv, s);
  return bwd_hd<T, 128>(g, qkv, dl, lse, delta, dqkv, s);
}

template cudaError_t launch_local_fwd_simt<float>(const Geom&, const float*, float*, float*, cudaStream_t);
template cudaError_t launch_local_fwd_simt<bf16>(const Geom&, const bf16*, bf16*, float*, cudaStream_t);
template cudaError_t launch_local_bwd_simt<float>(const Geom&, const float*, const float*, const float*,
                                                  const float*, float*, cudaStream_t);
template cudaError_t launch_local_bwd_simt<bf16>(const Geom&, const bf16*, const bf16*, const float*,
                                                 const float*, bf16*, cudaStream_t);

}  // namespace llattn
