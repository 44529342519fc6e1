// Latent branch: causal-chunk attention of latent query rows against the
// pooled chunk keys/values (models.py:361-375), forward and backward.
//
// rq [B,Tq,Lh,ldh], gkv [B,Nc,2,Lh,ldh] (gk = slot 0, gv = slot 1).
// Row r sees chunks j < qid(r); a row with qid = 0 outputs 0 (models.py:366-373).
// The work is tiny next to the local branch (Nc <= 512 keys of ldh <= 64), so
// these kernels use fp32 FMAs with the per-(b, latent head) keys staged in
// shared memory; ldh is padded with zeros up to the template width L.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace llattn {
namespace {

constexpr int kRowsFwd = 128;  // query rows per CTA (one thread each)
constexpr int kKeyTile = 64;   // chunk keys staged per shared-memory tile

template <typename T, int L>
__global__ void __launch_bounds__(kRowsFwd) latent_fwd_kernel(Geom g, const T* __restrict__ rq,
                                                              const T* __restrict__ gkv,
                                                              T* __restrict__ lat,
                                                              float* __restrict__ lat_lse) {
  __shared__ float sk[kKeyTile][L];
  __shared__ float sv[kKeyTile][L];
  const int b = blockIdx.z, lh = blockIdx.y;
  const int r = blockIdx.x * kRowsFwd + threadIdx.x;
  const bool valid = r < g.Tq;
  const int qid = valid ? row_qid(g, r) : 0;
  const int max_qid = row_qid(g, min((int)(blockIdx.x * kRowsFwd + kRowsFwd - 1), g.Tq - 1));

  float q[L];
#pragma unroll
  for (int e = 0; e < L; ++e) {
    q[e] = (valid && e < g.ldh)
               ? to_f<T>(rq[((int64_t)(b * g.Tq + r) * g.Lh + lh) * g.ldh + e]) * g.lat_scale
               : 0.f;
  }
  float m = -INFINITY, l = 0.f, acc[L];
#pragma unroll
  for (int e = 0; e < L; ++e) acc[e] = 0.f;

  for (int j0 = 0; j0 < max_qid; j0 += kKeyTile) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kKeyTile * L; idx += kRowsFwd) {
      const int jj = idx / L, e = idx % L, j = j0 + jj;
      float kv = 0.f, vv = 0.f;
      if (j < g.Nc && e < g.ldh) {
        const int64_t base = ((int64_t)(b * g.Nc + j) * 2 * g.Lh + lh) * g.ldh + e;
        kv = to_f<T>(gkv[base]);
        vv = to_f<T>(gkv[base + (int64_t)g.Lh * g.ldh]);
      }
      sk[jj][e] = kv;
      sv[jj][e] = vv;
    }
    __syncthreads();
    const int n = min(kKeyTile, qid - j0);
    for (int u0 = 0; u0 < n; u0 += 16) {
      float s[16];
      float mx = m;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < L; ++e) dot = fmaf(q[e], sk[u0 + u][e], dot);
        s[u] = (u0 + u < n) ? dot : -INFINITY;
        mx = fmaxf(mx, s[u]);
      }
      const float corr = expf(m - mx);  // m = -inf on the first tile -> 0
      l *= corr;
#pragma unroll
      for (int e = 0; e < L; ++e) acc[e] *= corr;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const float p = expf(s[u] - mx);
        l += p;
#pragma unroll
        for (int e = 0; e < L; ++e) acc[e] = fmaf(p, sv[u0 + u][e], acc[e]);
      }
      m = mx;
    }
  }
  if (!valid) return;
  const float inv = qid > 0 ? 1.f / l : 0.f;
  T* dst = lat + (int64_t)(b * g.Tq + r) * g.Ld + lh * g.ldh;
#pragma unroll
  for (int e = 0; e < L; ++e)
    if (e < g.ldh) dst[e] = from_f<T>(acc[e] * inv);
  lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r] = qid > 0 ? m + logf(l) : INFINITY;
}

// ---------------------------------------------------------------------------
// Backward. With P = softmax(s) (s = lat_scale * rq.gk), dP = dlat.gv,
// delta = dlat.lat, dS = P (dP - delta):
//   drq = lat_scale * sum_j dS gk_j,  dgk_j = lat_scale * sum_r dS rq_r,
//   dgv_j = sum_r P dlat_r.
// Kernel 1 (row-major CTAs) computes drq and delta. Kernel 2 (key-major CTAs,
// rows split in n_split ranges) accumulates dgk/dgv for 64 keys in registers
// and writes one partial per row range; a reduce sums the partials in a fixed
// order, so the result is deterministic.

constexpr int kRowsBwd = 64;

template <typename T, int L>
__global__ void __launch_bounds__(256) latent_bwd_rows_kernel(
    Geom g, const T* __restrict__ rq, const T* __restrict__ gkv, const T* __restrict__ lat,
    const float* __restrict__ lat_lse, const float* __restrict__ dlat, T* __restrict__ drq,
    float* __restrict__ delta_ws) {
  extern __shared__ float smem_rows[];
  float(*s_rq)[L + 1] = reinterpret_cast<float(*)[L + 1]>(smem_rows);
  float(*s_dl)[L + 1] = s_rq + kRowsBwd;
  float(*s_k)[L + 1] = s_dl + kRowsBwd;
  float(*s_v)[L + 1] = s_k + kKeyTile;
  float(*s_ds)[kKeyTile + 1] = reinterpret_cast<float(*)[kKeyTile + 1]>(s_v + kKeyTile);
  float* s_lse = reinterpret_cast<float*>(s_ds + kRowsBwd);
  float* s_delta = s_lse + kRowsBwd;
  int* s_qid = reinterpret_cast<int*>(s_delta + kRowsBwd);
  const int b = blockIdx.z, lh = blockIdx.y, r0 = blockIdx.x * kRowsBwd;
  const int tid = threadIdx.x;

  for (int idx = tid; idx < kRowsBwd * L; idx += 256) {
    const int i = idx / L, e = idx % L, r = r0 + i;
    float a = 0.f, dv = 0.f;
    if (r < g.Tq && e < g.ldh) {
      a = to_f<T>(rq[((int64_t)(b * g.Tq + r) * g.Lh + lh) * g.ldh + e]);
      dv = dlat[(int64_t)(b * g.Tq + r) * g.Ld + lh * g.ldh + e];
    }
    s_rq[i][e] = a;
    s_dl[i][e] = dv;
  }
  if (tid < kRowsBwd) {
    const int r = r0 + tid;
    if (r < g.Tq) {
      s_lse[tid] = lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r];
      s_qid[tid] = row_qid(g, r);
    } else {
      s_lse[tid] = INFINITY;
      s_qid[tid] = 0;
    }
  }
  const int max_qid = row_qid(g, min(r0 + kRowsBwd - 1, g.Tq - 1));
  // thread -> (row ri, 4-key subset kc) for dS; (row ri, e-subset ec) for drq
  const int ri = tid / 4, kc = tid % 4;
  constexpr int EPT = (L + 3) / 4;
  float acc[EPT];
#pragma unroll
  for (int u = 0; u < EPT; ++u) acc[u] = 0.f;

  // delta = dlat . lat, taken as sum_j P_j (dlat . gv_j) in fp32 rather than
  // from the stored (rounded) lat: with long chunks the pooled values are
  // nearly equal and dS = P (dlat.gv_j - delta) cancels, so delta must be
  // consistent with P to working precision
  float dpart = 0.f;
  for (int j0 = 0; j0 < max_qid; j0 += kKeyTile) {
    __syncthreads();
    for (int idx = tid; idx < kKeyTile * L; idx += 256) {
      const int jj = idx / L, e = idx % L, j = j0 + jj;
      float kv = 0.f, vv = 0.f;
      if (j < g.Nc && e < g.ldh) {
        const int64_t base = ((int64_t)(b * g.Nc + j) * 2 * g.Lh + lh) * g.ldh + e;
        kv = to_f<T>(gkv[base]);
        vv = to_f<T>(gkv[base + (int64_t)g.Lh * g.ldh]);
      }
      s_k[jj][e] = kv;
      s_v[jj][e] = vv;
    }
    __syncthreads();
    const float lse = s_lse[ri];
    const int qid = s_qid[ri];
    for (int u = 0; u < kKeyTile / 4; ++u) {
      const int jj = kc + 4 * u;
      if (j0 + jj < qid) {
        float sd = 0.f, dp = 0.f;
#pragma unroll
        for (int e = 0; e < L; ++e) {
          sd = fmaf(s_rq[ri][e], s_k[jj][e], sd);
          dp = fmaf(s_dl[ri][e], s_v[jj][e], dp);
        }
        dpart = fmaf(expf(sd * g.lat_scale - lse), dp, dpart);
      }
    }
  }
  dpart += __shfl_xor_sync(0xffffffffu, dpart, 1);
  dpart += __shfl_xor_sync(0xffffffffu, dpart, 2);
  if (kc == 0) {
    s_delta[ri] = dpart;
    if (r0 + ri < g.Tq) delta_ws[(int64_t)(b * g.Lh + lh) * g.Tq + r0 + ri] = dpart;
  }

  for (int j0 = 0; j0 < max_qid; j0 += kKeyTile) {
    __syncthreads();
    for (int idx = tid; idx < kKeyTile * L; idx += 256) {
      const int jj = idx / L, e = idx % L, j = j0 + jj;
      float kv = 0.f, vv = 0.f;
      if (j < g.Nc && e < g.ldh) {
        const int64_t base = ((int64_t)(b * g.Nc + j) * 2 * g.Lh + lh) * g.ldh + e;
        kv = to_f<T>(gkv[base]);
        vv = to_f<T>(gkv[base + (int64_t)g.Lh * g.ldh]);
      }
      s_k[jj][e] = kv;
      s_v[jj][e] = vv;
    }
    __syncthreads();
    {
      const float lse = s_lse[ri], dlt = s_delta[ri];
      const int qid = s_qid[ri];
#pragma unroll 4
      for (int u = 0; u < kKeyTile / 4; ++u) {
        const int jj = kc + 4 * u;
        float sd = 0.f, dp = 0.f;
#pragma unroll
        for (int e = 0; e < L; ++e) {
          sd = fmaf(s_rq[ri][e], s_k[jj][e], sd);
          dp = fmaf(s_dl[ri][e], s_v[jj][e], dp);
        }
        float ds = 0.f;
        if (j0 + jj < qid) {
          const float p = expf(sd * g.lat_scale - lse);
          ds = p * (dp - dlt);
        }
        s_ds[ri][jj] = ds;
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < EPT; ++u) {
      const int e = kc + 4 * u;
      if (e < L) {
        float a = acc[u];
        for (int jj = 0; jj < kKeyTile; ++jj) a = fmaf(s_ds[ri][jj], s_k[jj][e], a);
        acc[u] = a;
      }
    }
  }
  const int r = r0 + ri;
  if (r < g.Tq) {
#pragma unroll
    for (int u = 0; u < EPT; ++u) {
      const int e = kc + 4 * u;
      if (e < g.ldh)
        drq[((int64_t)(b * g.Tq + r) * g.Lh + lh) * g.ldh + e] = from_f<T>(acc[u] * g.lat_scale);
    }
  }
}

constexpr int kRowsSub = 32;  // rows per inner step of the key-major kernel

template <typename T, int L>
__global__ void __launch_bounds__(256) latent_bwd_keys_kernel(
    Geom g, const T* __restrict__ rq, const T* __restrict__ gkv, const float* __restrict__ lat_lse,
    const float* __restrict__ dlat, const float* __restrict__ delta_ws, float* __restrict__ part,
    int n_split) {
  extern __shared__ float smem_keys[];
  float(*s_k)[L + 1] = reinterpret_cast<float(*)[L + 1]>(smem_keys);
  float(*s_v)[L + 1] = s_k + kKeyTile;
  float(*s_rq)[L + 1] = s_v + kKeyTile;
  float(*s_dl)[L + 1] = s_rq + kRowsSub;
  float(*s_p)[kKeyTile + 1] = reinterpret_cast<float(*)[kKeyTile + 1]>(s_dl + kRowsSub);
  float(*s_ds)[kKeyTile + 1] = s_p + kRowsSub;
  float* s_lse = reinterpret_cast<float*>(s_ds + kRowsSub);
  float* s_delta = s_lse + kRowsSub;
  int* s_qid = reinterpret_cast<int*>(s_delta + kRowsSub);
  const int tid = threadIdx.x;
  const int n_ktiles = cdiv(g.Nc, kKeyTile);
  const int kt = blockIdx.x % n_ktiles, split = blockIdx.x / n_ktiles;
  const int b = blockIdx.z, lh = blockIdx.y, j0 = kt * kKeyTile;

  for (int idx = tid; idx < kKeyTile * L; idx += 256) {
    const int jj = idx / L, e = idx % L, j = j0 + jj;
    float kv = 0.f, vv = 0.f;
    if (j < g.Nc && e < g.ldh) {
      const int64_t base = ((int64_t)(b * g.Nc + j) * 2 * g.Lh + lh) * g.ldh + e;
      kv = to_f<T>(gkv[base]);
      vv = to_f<T>(gkv[base + (int64_t)g.Lh * g.ldh]);
    }
    s_k[jj][e] = kv;
    s_v[jj][e] = vv;
  }
  // rows that can see chunk j0: qid(r) > j0. qid is non-decreasing in r, so
  // that is a suffix [r_first, Tq); find it by bisection.
  int lo = 0, hi = g.Tq;
  while (lo < hi) {
    const int mid = (lo + hi) / 2;
    if (row_qid(g, mid) > j0) hi = mid; else lo = mid + 1;
  }
  const int r_first = lo;
  const int n_rows = g.Tq - r_first;
  const int per = cdiv(cdiv(max(n_rows, 1), n_split), kRowsSub) * kRowsSub;
  const int ra = r_first + split * per, rb = min(g.Tq, ra + per);

  // accumulators: key jk = tid/4, e-subset ec = tid%4
  const int jk = tid / 4, ec = tid % 4;
  constexpr int EPT = (L + 3) / 4;
  float agk[EPT], agv[EPT];
#pragma unroll
  for (int u = 0; u < EPT; ++u) agk[u] = agv[u] = 0.f;

  for (int rs = ra; rs < rb; rs += kRowsSub) {
    __syncthreads();
    for (int idx = tid; idx < kRowsSub * L; idx += 256) {
      const int i = idx / L, e = idx % L, r = rs + i;
      float a = 0.f, dv = 0.f;
      if (r < rb && e < g.ldh) {
        a = to_f<T>(rq[((int64_t)(b * g.Tq + r) * g.Lh + lh) * g.ldh + e]);
        dv = dlat[(int64_t)(b * g.Tq + r) * g.Ld + lh * g.ldh + e];
      }
      s_rq[i][e] = a;
      s_dl[i][e] = dv;
    }
    if (tid < kRowsSub) {
      const int r = rs + tid;
      if (r < rb) {
        s_lse[tid] = lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r];
        s_delta[tid] = delta_ws[(int64_t)(b * g.Lh + lh) * g.Tq + r];
        s_qid[tid] = row_qid(g, r);
      } else {
        s_lse[tid] = INFINITY;
        s_delta[tid] = 0.f;
        s_qid[tid] = 0;
      }
    }
    __syncthreads();
    // 32 rows x 64 keys = 2048 pairs, 8 per thread: row = tid/8, key = tid%8 + 8u
    {
      const int ri = tid / 8, kc = tid % 8;
      const float lse = s_lse[ri], dlt = s_delta[ri];
      const int qid = s_qid[ri];
#pragma unroll
      for (int u = 0; u < kKeyTile / 8; ++u) {
        const int jj = kc + 8 * u;
        float sd = 0.f, dp = 0.f;
#pragma unroll
        for (int e = 0; e < L; ++e) {
          sd = fmaf(s_rq[ri][e], s_k[jj][e], sd);
          dp = fmaf(s_dl[ri][e], s_v[jj][e], dp);
        }
        float p = 0.f, ds = 0.f;
        if (j0 + jj < qid) {
          p = expf(sd * g.lat_scale - lse);
          ds = p * (dp - dlt);
        }
        s_p[ri][jj] = p;
        s_ds[ri][jj] = ds;
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < EPT; ++u) {
      const int e = ec + 4 * u;
      if (e < L) {
        float a = agk[u], v = agv[u];
        for (int i = 0; i < kRowsSub; ++i) {
          a = fmaf(s_ds[i][jk], s_rq[i][e], a);
          v = fmaf(s_p[i][jk], s_dl[i][e], v);
        }
        agk[u] = a;
        agv[u] = v;
      }
    }
  }
  const int j = j0 + jk;
  if (j < g.Nc) {
    float* dst = part + (int64_t)split * g.B * g.Nc * 2 * g.Ld;
#pragma unroll
    for (int u = 0; u < EPT; ++u) {
      const int e = ec + 4 * u;
      if (e < g.ldh) {
        const int64_t base = ((int64_t)(b * g.Nc + j) * 2 * g.Lh + lh) * g.ldh + e;
        dst[base] = agk[u] * g.lat_scale;
        dst[base + (int64_t)g.Lh * g.ldh] = agv[u];
      }
    }
  }
}

template <typename To>
__global__ void reduce_parts_kernel(const float* __restrict__ part, int n_part, int64_t n,
                                    To* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float a = 0.f;
    for (int p = 0; p < n_part; ++p) a += part[(int64_t)p * n + i];
    out[i] = from_f<To>(a);
  }
}

template <typename T, int L>
cudaError_t latent_fwd_l(const Geom& g, const T* rq, const T* gkv, T* lat, float* lse, cudaStream_t s) {
  dim3 grid(cdiv(g.Tq, kRowsFwd), g.Lh, g.B);
  latent_fwd_kernel<T, L><<<grid, kRowsFwd, 0, s>>>(g, rq, gkv, lat, lse);
  return cudaGetLastError();
}

template <typename T, int L>
cudaError_t latent_bwd_l(const Geom& g, const T* rq, const T* gkv, const T* lat, const float* lse,
                         const float* dlat, T* drq, float* part, int n_split, float* delta,
                         cudaStream_t s) {
  const size_t sm1 = sizeof(float) * ((2 * kRowsBwd + 2 * kKeyTile) * (L + 1) +
                                      kRowsBwd * (kKeyTile + 1) + 3 * kRowsBwd);
  const size_t sm2 = sizeof(float) * ((2 * kKeyTile + 2 * kRowsSub) * (L + 1) +
                                      2 * kRowsSub * (kKeyTile + 1) + 3 * kRowsSub);
  cudaError_t e = cudaFuncSetAttribute(latent_bwd_rows_kernel<T, L>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(latent_bwd_keys_kernel<T, L>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2);
  if (e != cudaSuccess) return e;
  dim3 g1(cdiv(g.Tq, kRowsBwd), g.Lh, g.B);
  latent_bwd_rows_kernel<T, L><<<g1, 256, sm1, s>>>(g, rq, gkv, lat, lse, dlat, drq, delta);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  dim3 g2(cdiv(g.Nc, kKeyTile) * n_split, g.Lh, g.B);
  latent_bwd_keys_kernel<T, L><<<g2, 256, sm2, s>>>(g, rq, gkv, lse, dlat, delta, part, n_split);
  return cudaGetLastError();
}

}  // namespace

template <typename T>
cudaError_t launch_latent_fwd(const Geom& g, const T* rq, const T* gkv, T* lat, float* lat_lse,
                              cudaStream_t s) {
  if (g.ldh <= 8) return latent_fwd_l<T, 8>(g, rq, gkv, lat, lat_lse, s);
  if (g.ldh <= 16) return latent_fwd_l<T, 16>(g, rq, gkv, lat, lat_lse, s);
  if (g.ldh <= 32) return latent_fwd_l<T, 32>(g, rq, gkv, lat, lat_lse, s);
  return latent_fwd_l<T, 64>(g, rq, gkv, lat, lat_lse, s);
}

template <typename T>
cudaError_t launch_latent_bwd(const Geom& g, const T* rq, const T* gkv, const T* lat,
                              const float* lat_lse, const float* dlat, T* drq, float* dgkv_part,
                              int n_split, float* delta_ws, cudaStream_t s) {
  if (g.ldh <= 8)
    return latent_bwd_l<T, 8>(g, rq, gkv, lat, lat_lse, dlat, drq, dgkv_part, n_split, delta_ws, s);
  if (g.ldh <= 16)
    return latent_bwd_l<T, 16>(g, rq, gkv, lat, lat_lse, dlat, drq, dgkv_part, n_split, delta_ws, s);
  if (g.ldh <= 32)
    return latent_bwd_l<T, 32>(g, rq, gkv, lat, lat_lse, dlat, drq, dgkv_part, n_split, delta_ws, s);
  return latent_bwd_l<T, 64>(g, rq, gkv, lat, lat_lse, dlat, drq, dgkv_part, n_split, delta_ws, s);
}

template <typename T>
cudaError_t launch_latent_reduce(const Geom& g, const float* part, int n_split, T* dgkv,
                                 cudaStream_t s) {
  const int64_t n = (int64_t)g.B * g.Nc * 2 * g.Ld;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  reduce_parts_kernel<T><<<blocks, 256, 0, s>>>(part, n_split, n, dgkv);
  return cudaGetLastError();
}

cudaError_t launch_reduce_rows(const float* part, int n_part, int64_t n, float* out, cudaStream_t s) {
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  reduce_parts_kernel<float><<<blocks, 256, 0, s>>>(part, n_part, n, out);
  return cudaGetLastError();
}

template cudaError_t launch_latent_fwd<float>(const Geom&, const float*, const float*, float*, float*, cudaStream_t);
template cudaError_t launch_latent_fwd<bf16>(const Geom&, const bf16*, const bf16*, bf16*, float*, cudaStream_t);
template cudaError_t launch_latent_bwd<float>(const Geom&, const float*, const float*, const float*, const float*,
                                              const float*, float*, float*, int, float*, cudaStream_t);
template cudaError_t launch_latent_bwd<bf16>(const Geom&, const bf16*, const bf16*, const bf16*, const float*,
                                             const float*, bf16*, float*, int, float*, cudaStream_t);
template cudaError_t launch_latent_reduce<float>(const Geom&, const float*, int, float*, cudaStream_t);
template cudaError_t launch_latent_reduce<bf16>(const Geom&, const float*, int, bf16*, cudaStream_t);

}  // namespace llattn
