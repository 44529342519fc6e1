// Remote projection, gate and mix (models.py:392-438), forward and backward,
// plus the backward of the r_out projection. Exact fp32 path (SIMT FMAs).
//
//   remote[t] = lat[row(t)] W_rout^T + b_rout            (row(t) = t / qbs)
//   w_h       = sigmoid(local_h.g_l + gate_bias - remote_h.g_r)
//   mixed_h   = w_h local_h + (1 - w_h) remote_h
// Backward, per token and head, with dm = dmixed_h:
//   ds = (dm.(local_h - remote_h)) w (1 - w)
//   dlocal  = w dm + ds g_l          (written for the local-branch backward)
//   dremote = (1 - w) dm - ds g_r    (fp32, reduced over query blocks later)
//   dg_l += ds local_h,  dg_r -= ds remote_h
//   D_h = dlocal.local_h             (the local backward's row term)
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace llattn {
namespace {

constexpr int NT = 128;

template <typename T>
__device__ __forceinline__ void remote_row(const Geom& g, const float* slat, const T* __restrict__ w_rout,
                                           const float* __restrict__ b_rout, float* sR) {
  for (int c = threadIdx.x; c < g.d; c += NT) {
    const T* wr = w_rout + (int64_t)c * g.Ld;
    float a = b_rout[c];
    for (int k = 0; k < g.Ld; ++k) a = fmaf(slat[k], to_f<T>(wr[k]), a);
    sR[c] = a;
  }
}

template <typename T>
__global__ void __launch_bounds__(NT) gate_fwd_kernel(Geom g, const T* __restrict__ local_out,
                                                      const T* __restrict__ lat,
                                                      const T* __restrict__ w_rout,
                                                      const float* __restrict__ b_rout,
                                                      const float* __restrict__ gl,
                                                      const float* __restrict__ gr,
                                                      T* __restrict__ mixed) {
  extern __shared__ float smem_gf[];
  float* sR = smem_gf;
  float* sL = sR + g.d;
  float* slat = sL + g.d;
  float* sw = slat + g.Ld;
  const int t = blockIdx.x, b = blockIdx.y, r = t / g.qbs;
  const int64_t row = (int64_t)b * g.T + t;
  for (int k = threadIdx.x; k < g.Ld; k += NT) slat[k] = to_f<T>(lat[((int64_t)b * g.Tq + r) * g.Ld + k]);
  for (int c = threadIdx.x; c < g.d; c += NT) sL[c] = to_f<T>(local_out[row * g.d + c]);
  __syncthreads();
  remote_row<T>(g, slat, w_rout, b_rout, sR);
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int h = warp; h < g.H; h += NT / 32) {
    float sl = 0.f, sr = 0.f;
    for (int e = lane; e < g.hd; e += 32) {
      sl = fmaf(sL[h * g.hd + e], gl[e], sl);
      sr = fmaf(sR[h * g.hd + e], gr[e], sr);
    }
    sl = warp_sum(sl);
    sr = warp_sum(sr);
    if (lane == 0) {
      // both weights computed directly: 1 - w would lose the small one's
      // precision when the gate saturates
      const float x = sl + g.gate_bias - sr;
      sw[2 * h] = 1.f / (1.f + expf(-x));
      sw[2 * h + 1] = 1.f / (1.f + expf(x));
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < g.d; c += NT) {
    const int h = c / g.hd;
    mixed[row * g.d + c] = from_f<T>(sw[2 * h] * sL[c] + sw[2 * h + 1] * sR[c]);
  }
}

template <typename T>
__global__ void __launch_bounds__(NT) gate_bwd_kernel(
    Geom g, const T* __restrict__ local_out, const T* __restrict__ lat, const T* __restrict__ w_rout,
    const float* __restrict__ b_rout, const float* __restrict__ gl, const float* __restrict__ gr,
    const T* __restrict__ dmixed, T* __restrict__ dl, float* __restrict__ delta,
    float* __restrict__ drow, float* __restrict__ dg_part, int tok_per_cta) {
  extern __shared__ float smem_gb[];
  float* sR = smem_gb;
  float* sL = sR + g.d;
  float* sdm = sL + g.d;
  float* slat = sdm + g.d;
  float* sds = slat + g.Ld;
  const int b = blockIdx.y;
  const int ta = blockIdx.x * tok_per_cta, tb = min(g.T, ta + tok_per_cta);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float agl = 0.f, agr = 0.f;  // thread e = threadIdx.x (hd <= 128)
  for (int t = ta; t < tb; ++t) {
    const int r = t / g.qbs;
    const int64_t row = (int64_t)b * g.T + t;
    __syncthreads();
    for (int k = threadIdx.x; k < g.Ld; k += NT) slat[k] = to_f<T>(lat[((int64_t)b * g.Tq + r) * g.Ld + k]);
    for (int c = threadIdx.x; c < g.d; c += NT) {
      sL[c] = to_f<T>(local_out[row * g.d + c]);
      sdm[c] = to_f<T>(dmixed[row * g.d + c]);
    }
    __syncthreads();
    remote_row<T>(g, slat, w_rout, b_rout, sR);
    __syncthreads();
    for (int h = warp; h < g.H; h += NT / 32) {
      const float* L = sL + h * g.hd;
      const float* R = sR + h * g.hd;
      const float* dm = sdm + h * g.hd;
      float sl = 0.f, sr = 0.f, dw = 0.f;
      for (int e = lane; e < g.hd; e += 32) {
        sl = fmaf(L[e], gl[e], sl);
        sr = fmaf(R[e], gr[e], sr);
        dw = fmaf(dm[e], L[e] - R[e], dw);
      }
      sl = warp_sum(sl);
      sr = warp_sum(sr);
      dw = warp_sum(dw);
      const float x = sl + g.gate_bias - sr;
      const float w = 1.f / (1.f + expf(-x));
      const float wr = 1.f / (1.f + expf(x));
      const float ds = dw * w * wr;
      float dsum = 0.f;
      for (int e = lane; e < g.hd; e += 32) {
        const float dlv = w * dm[e] + ds * gl[e];
        const T dlt = from_f<T>(dlv);
        dl[row * g.d + h * g.hd + e] = dlt;
        dsum = fmaf(to_f<T>(dlt), L[e], dsum);
        drow[row * g.d + h * g.hd + e] = wr * dm[e] - ds * gr[e];
      }
      dsum = warp_sum(dsum);
      if (lane == 0) {
        sds[h] = ds;
        delta[((int64_t)b * g.H + h) * g.T + t] = dsum;
      }
    }
    __syncthreads();
    if (threadIdx.x < g.hd) {
      const int e = threadIdx.x;
      for (int h = 0; h < g.H; ++h) {
        agl = fmaf(sds[h], sL[h * g.hd + e], agl);
        agr = fmaf(-sds[h], sR[h * g.hd + e], agr);
      }
    }
  }
  if (threadIdx.x < g.hd) {
    float* dst = dg_part + ((int64_t)b * gridDim.x + blockIdx.x) * 2 * g.hd;
    dst[threadIdx.x] = agl;
    dst[g.hd + threadIdx.x] = agr;
  }
}

// dlat[row] = (sum over the row's tokens of dremote) . W_rout
template <int LM>
__global__ void __launch_bounds__(256) rout_dlat_kernel(Geom g, const float* __restrict__ drow,
                                                        const void* __restrict__ w_rout_v, int w_bf16,
                                                        float* __restrict__ dlat) {
  extern __shared__ float smem_rd[];
  float(*sdr)[64 + 1] = reinterpret_cast<float(*)[64 + 1]>(smem_rd);  // [32 rows][64 c]
  float(*sw)[LM + 1] = reinterpret_cast<float(*)[LM + 1]>(sdr + 32);  // [64 c][LM]
  const int tid = threadIdx.x, ri = tid / 8, kg = tid % 8;
  const int R0 = blockIdx.x * 32;  // flattened (b, r) rows
  const int n_rows = g.B * g.Tq;
  float acc[LM / 8];
#pragma unroll
  for (int u = 0; u < LM / 8; ++u) acc[u] = 0.f;
  for (int c0 = 0; c0 < g.d; c0 += 64) {
    __syncthreads();
    for (int idx = tid; idx < 32 * 64; idx += 256) {
      const int i = idx / 64, cc = idx % 64, R = R0 + i, c = c0 + cc;
      float a = 0.f;
      if (R < n_rows && c < g.d) {
        const int b = R / g.Tq, r = R % g.Tq;
        const int t1 = min(g.T, (r + 1) * g.qbs);
        for (int t = r * g.qbs; t < t1; ++t) a += drow[((int64_t)b * g.T + t) * g.d + c];
      }
      sdr[i][cc] = a;
    }
    for (int idx = tid; idx < 64 * LM; idx += 256) {
      const int cc = idx / LM, k = idx % LM, c = c0 + cc;
      float v = 0.f;
      if (c < g.d && k < g.Ld) {
        const int64_t o = (int64_t)c * g.Ld + k;
        v = w_bf16 ? __bfloat162float(reinterpret_cast<const bf16*>(w_rout_v)[o])
                   : reinterpret_cast<const float*>(w_rout_v)[o];
      }
      sw[cc][k] = v;
    }
    __syncthreads();
    for (int cc = 0; cc < 64; ++cc) {
      const float a = sdr[ri][cc];
#pragma unroll
      for (int u = 0; u < LM / 8; ++u) acc[u] = fmaf(a, sw[cc][kg + 8 * u], acc[u]);
    }
  }
  const int R = R0 + ri;
  if (R < n_rows) {
#pragma unroll
    for (int u = 0; u < LM / 8; ++u) {
      const int k = kg + 8 * u;
      if (k < g.Ld) dlat[(int64_t)R * g.Ld + k] = acc[u];
    }
  }
}

// partial dW_rout[c, k] and db_rout[c] over one split of the (b, r) rows.
template <typename T, int LM>
__global__ void __launch_bounds__(256) rout_dw_kernel(Geom g, const float* __restrict__ drow,
                                                      const T* __restrict__ lat,
                                                      float* __restrict__ dw_part,
                                                      float* __restrict__ db_part, int n_split) {
  __shared__ float sdr[32][32 + 1];
  __shared__ float sl[32][LM + 1];
  const int tid = threadIdx.x, ci = tid / 8, kg = tid % 8;
  const int c0 = blockIdx.x * 32, split = blockIdx.y;
  const int n_rows = g.B * g.Tq;
  const int per = cdiv(cdiv(n_rows, n_split), 32) * 32;
  const int Ra = split * per, Rb = min(n_rows, Ra + per);
  float acc[LM / 8], adb = 0.f;
#pragma unroll
  for (int u = 0; u < LM / 8; ++u) acc[u] = 0.f;
  for (int R0 = Ra; R0 < Rb; R0 += 32) {
    __syncthreads();
    for (int idx = tid; idx < 32 * 32; idx += 256) {
      const int i = idx / 32, cc = idx % 32, R = R0 + i, c = c0 + cc;
      float a = 0.f;
      if (R < Rb && c < g.d) {
        const int b = R / g.Tq, r = R % g.Tq;
        const int t1 = min(g.T, (r + 1) * g.qbs);
        for (int t = r * g.qbs; t < t1; ++t) a += drow[((int64_t)b * g.T + t) * g.d + c];
      }
      sdr[i][cc] = a;
    }
    for (int idx = tid; idx < 32 * LM; idx += 256) {
      const int i = idx / LM, k = idx % LM, R = R0 + i;
      sl[i][k] = (R < Rb && k < g.Ld) ? to_f<T>(lat[(int64_t)R * g.Ld + k]) : 0.f;
    }
    __syncthreads();
    for (int i = 0; i < 32; ++i) {
      const float a = sdr[i][ci];
      adb += a;
#pragma unroll
      for (int u = 0; u < LM / 8; ++u) acc[u] = fmaf(a, sl[i][kg + 8 * u], acc[u]);
    }
  }
  const int c = c0 + ci;
  if (c < g.d) {
    float* dst = dw_part + (int64_t)split * g.d * g.Ld + (int64_t)c * g.Ld;
#pragma unroll
    for (int u = 0; u < LM / 8; ++u) {
      const int k = kg + 8 * u;
      if (k < g.Ld) dst[k] = acc[u];
    }
    if (kg == 0) db_part[(int64_t)split * g.d + c] = adb;
  }
}

template <typename T, int LM>
cudaError_t rout_bwd_lm(const Geom& g, const float* drow, const T* lat, const T* w_rout, float* dlat,
                        float* dw_part, int n_split, cudaStream_t s) {
  const size_t sm = sizeof(float) * (32 * 65 + 64 * (LM + 1));
  cudaError_t e = set_smem_once(rout_dlat_kernel<LM>, (int)sm);
  if (e != cudaSuccess) return e;
  const int n_rows = g.B * g.Tq;
  rout_dlat_kernel<LM><<<cdiv(n_rows, 32), 256, sm, s>>>(g, drow, w_rout, sizeof(T) == 2, dlat);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  float* db_part = dw_part + (int64_t)n_split * g.d * g.Ld;
  dim3 grid(cdiv(g.d, 32), n_split);
  rout_dw_kernel<T, LM><<<grid, 256, 0, s>>>(g, drow, lat, dw_part, db_part, n_split);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// Gate and mix with the remote projection precomputed (bf16, any latent
// width): the tensor-core GEMM writes remote = lat W_rout^T + b_rout, these
// kernels do the per-(token, head) gate arithmetic, one warp per (token,
// head) pair with 4 elements per lane (head_dim <= 128, a multiple of 4).
// A CTA covers RM_TOK tokens (token-wise latent queries) or one query block
// (block-pooled ones); warp w takes the heads h = w mod 8 of every token, so
// a head's running sums stay in one warp and the order of every sum is fixed.

constexpr int RM_WARPS = 8, RM_TOK = 16;

__device__ __forceinline__ void ld4(const bf16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  v[0] = __uint_as_float(u.x << 16);
  v[1] = __uint_as_float(u.x & 0xffff0000u);
  v[2] = __uint_as_float(u.y << 16);
  v[3] = __uint_as_float(u.y & 0xffff0000u);
}
__device__ __forceinline__ void st4(bf16* p, const float (&v)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// mixed holds the remote rows on entry: token t's at row t (token-wise), or
// query block r's at the block's first row r * qbs (read by this CTA alone,
// into shared memory, before any of the block's rows is overwritten).
__global__ void __launch_bounds__(RM_WARPS * 32) gate_mix_rmem_kernel(Geom g, const bf16* __restrict__ local_out,
                                                                     const float* __restrict__ gl,
                                                                     const float* __restrict__ gr,
                                                                     bf16* __restrict__ mixed) {
  extern __shared__ __align__(16) bf16 srem[];  // block-pooled queries: the block's remote row [d]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, b = blockIdx.y;
  const bool pooled = g.qbs > 1;
  const int ta = pooled ? blockIdx.x * g.qbs : blockIdx.x * RM_TOK;
  const int tb = min(g.T, ta + (pooled ? g.qbs : RM_TOK));
  if (pooled) {
    const uint4* src = reinterpret_cast<const uint4*>(mixed + ((int64_t)b * g.T + ta) * g.d);
    for (int i = threadIdx.x; i < g.d / 8; i += blockDim.x) reinterpret_cast<uint4*>(srem)[i] = src[i];
    __syncthreads();
  }
  const int e = 4 * lane;
  const bool on = e < g.hd;
  float vgl[4] = {0.f, 0.f, 0.f, 0.f}, vgr[4] = {0.f, 0.f, 0.f, 0.f};
  if (on) {
    const float4 a = *reinterpret_cast<const float4*>(gl + e), c = *reinterpret_cast<const float4*>(gr + e);
    vgl[0] = a.x; vgl[1] = a.y; vgl[2] = a.z; vgl[3] = a.w;
    vgr[0] = c.x; vgr[1] = c.y; vgr[2] = c.z; vgr[3] = c.w;
  }
  for (int t = ta; t < tb; ++t) {
    const int64_t row = (int64_t)b * g.T + t;
    for (int h = warp; h < g.H; h += RM_WARPS) {
      const int64_t o = row * g.d + (int64_t)h * g.hd + e;
      float L[4] = {0.f, 0.f, 0.f, 0.f}, R[4] = {0.f, 0.f, 0.f, 0.f};
      if (on) {
        ld4(local_out + o, L);
        ld4(pooled ? srem + h * g.hd + e : mixed + o, R);
      }
      float sl = 0.f, sr = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        sl = fmaf(L[k], vgl[k], sl);
        sr = fmaf(R[k], vgr[k], sr);
      }
      sl = warp_sum(sl);
      sr = warp_sum(sr);
      // both weights directly: 1 - w would lose the small one when the gate saturates
      const float x = sl + g.gate_bias - sr;
      const float w = 1.f / (1.f + expf(-x)), wr = 1.f / (1.f + expf(x));
      if (on) {
        float m[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) m[k] = w * L[k] + wr * R[k];
        st4(mixed + o, m);
      }
    }
  }
}

// Backward with the remote rows R [B*Tq, d] precomputed. Writes dl (bf16),
// the local backward's row term D = dl.local, the gradient of the remote
// projection's output (bf16; per token, or summed over each query block when
// the queries are block-pooled: the rows the r_out GEMMs take) and per-CTA
// gate partials dg_part[cta] = [sum ds local (hd), -sum ds remote (hd)].
__global__ void __launch_bounds__(RM_WARPS * 32) gate_bwd_rmem_kernel(
    Geom g, const bf16* __restrict__ local_out, const bf16* __restrict__ rem, const float* __restrict__ gl,
    const float* __restrict__ gr, const bf16* __restrict__ dmixed, bf16* __restrict__ dl,
    float* __restrict__ delta, bf16* __restrict__ dr, float* __restrict__ dg_part) {
  extern __shared__ __align__(16) float sgb[];  // [RM_WARPS][2 hd] partials, then (pooled) dR sums [d]
  float* sred = sgb;
  float* sdr = sgb + RM_WARPS * 2 * g.hd;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, b = blockIdx.y;
  const bool pooled = g.qbs > 1;
  const int ta = pooled ? blockIdx.x * g.qbs : blockIdx.x * RM_TOK;
  const int tb = min(g.T, ta + (pooled ? g.qbs : RM_TOK));
  const int e = 4 * lane;
  const bool on = e < g.hd;
  float vgl[4] = {0.f, 0.f, 0.f, 0.f}, vgr[4] = {0.f, 0.f, 0.f, 0.f};
  if (on) {
    const float4 a = *reinterpret_cast<const float4*>(gl + e), c = *reinterpret_cast<const float4*>(gr + e);
    vgl[0] = a.x; vgl[1] = a.y; vgl[2] = a.z; vgl[3] = a.w;
    vgr[0] = c.x; vgr[1] = c.y; vgr[2] = c.z; vgr[3] = c.w;
  }
  float agl[4] = {0.f, 0.f, 0.f, 0.f}, agr[4] = {0.f, 0.f, 0.f, 0.f};
  for (int h = warp; h < g.H; h += RM_WARPS) {
    float dsum[4] = {0.f, 0.f, 0.f, 0.f};  // pooled: this head's dR summed over the block
    for (int t = ta; t < tb; ++t) {
      const int64_t row = (int64_t)b * g.T + t;
      const int64_t o = row * g.d + (int64_t)h * g.hd + e;
      const int64_t orem = ((int64_t)b * g.Tq + t / g.qbs) * g.d + (int64_t)h * g.hd + e;
      float L[4] = {0.f, 0.f, 0.f, 0.f}, R[4] = {0.f, 0.f, 0.f, 0.f}, dm[4] = {0.f, 0.f, 0.f, 0.f};
      if (on) {
        ld4(local_out + o, L);
        ld4(rem + orem, R);
        ld4(dmixed + o, dm);
      }
      float sl = 0.f, sr = 0.f, dw = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        sl = fmaf(L[k], vgl[k], sl);
        sr = fmaf(R[k], vgr[k], sr);
        dw = fmaf(dm[k], L[k] - R[k], dw);
      }
      sl = warp_sum(sl);
      sr = warp_sum(sr);
      dw = warp_sum(dw);
      const float x = sl + g.gate_bias - sr;
      const float w = 1.f / (1.f + expf(-x)), wr = 1.f / (1.f + expf(x));
      const float ds = dw * w * wr;
      float dlv[4], drv[4], dd = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        dlv[k] = __bfloat162float(__float2bfloat16_rn(w * dm[k] + ds * vgl[k]));
        dd = fmaf(dlv[k], L[k], dd);
        drv[k] = wr * dm[k] - ds * vgr[k];
        agl[k] = fmaf(ds, L[k], agl[k]);
        agr[k] = fmaf(-ds, R[k], agr[k]);
      }
      dd = warp_sum(dd);
      if (on) {
        st4(dl + o, dlv);
        if (pooled) {
#pragma unroll
          for (int k = 0; k < 4; ++k) dsum[k] += drv[k];
        } else {
          st4(dr + o, drv);
        }
      }
      if (lane == 0) delta[((int64_t)b * g.H + h) * g.T + t] = dd;
    }
    if (pooled && on) st4(dr + ((int64_t)b * g.Tq + blockIdx.x) * g.d + (int64_t)h * g.hd + e, dsum);
  }
  if (on) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      sred[warp * 2 * g.hd + e + k] = agl[k];
      sred[warp * 2 * g.hd + g.hd + e + k] = agr[k];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * g.hd; i += blockDim.x) {
    float a = 0.f;
    for (int w = 0; w < RM_WARPS; ++w) a += sred[w * 2 * g.hd + i];
    dg_part[((int64_t)b * gridDim.x + blockIdx.x) * 2 * g.hd + i] = a;
  }
  (void)sdr;
}

}  // namespace

int gate_rmem_ctas(const Geom& g) { return g.B * (g.qbs > 1 ? g.Tq : cdiv(g.T, RM_TOK)); }

cudaError_t launch_gate_mix_rmem(const Geom& g, const bf16* local_out, const float* g_local, const float* g_remote,
                                 bf16* mixed, cudaStream_t s) {
  const size_t sm = g.qbs > 1 ? sizeof(bf16) * g.d : 0;
  if (sm > 48 * 1024) {
    cudaError_t e = set_smem_once(gate_mix_rmem_kernel, (int)sm);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(g.qbs > 1 ? g.Tq : cdiv(g.T, RM_TOK), g.B);
  gate_mix_rmem_kernel<<<grid, RM_WARPS * 32, sm, s>>>(g, local_out, g_local, g_remote, mixed);
  return cudaGetLastError();
}

cudaError_t launch_gate_bwd_rmem(const Geom& g, const bf16* local_out, const bf16* rem, const float* g_local,
                                 const float* g_remote, const bf16* dmixed, bf16* dl, float* delta, bf16* dr,
                                 float* dg_part, cudaStream_t s) {
  const size_t sm = sizeof(float) * RM_WARPS * 2 * g.hd;
  dim3 grid(g.qbs > 1 ? g.Tq : cdiv(g.T, RM_TOK), g.B);
  gate_bwd_rmem_kernel<<<grid, RM_WARPS * 32, sm, s>>>(g, local_out, rem, g_local, g_remote, dmixed, dl, delta, dr,
                                                       dg_part);
  return cudaGetLastError();
}


template <typename T>
cudaError_t launch_gate_fwd(const Geom& g, const T* local_out, const T* lat, const T* w_rout,
                            const float* b_rout, const float* g_local, const float* g_remote, T* mixed,
                            cudaStream_t s) {
  const size_t sm = sizeof(float) * (2 * g.d + g.Ld + 2 * g.H);
  cudaError_t e = set_smem_once(gate_fwd_kernel<T>, (int)sm);
  if (e != cudaSuccess) return e;
  dim3 grid(g.T, g.B);
  gate_fwd_kernel<T><<<grid, NT, sm, s>>>(g, local_out, lat, w_rout, b_rout, g_local, g_remote, mixed);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_gate_bwd(const Geom& g, const T* local_out, const T* lat, const T* w_rout,
                            const float* b_rout, const float* g_local, const float* g_remote,
                            const T* dmixed, T* dl, float* delta, float* drow, float* dg_part,
                            int tok_per_cta, cudaStream_t s) {
  const size_t sm = sizeof(float) * (3 * g.d + g.Ld + g.H);
  cudaError_t e = set_smem_once(gate_bwd_kernel<T>, (int)sm);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, tok_per_cta), g.B);
  gate_bwd_kernel<T><<<grid, NT, sm, s>>>(g, local_out, lat, w_rout, b_rout, g_local, g_remote, dmixed, dl,
                                          delta, drow, dg_part, tok_per_cta);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_rout_bwd(const Geom& g, const float* drow, const T* lat, const T* w_rout, float* dlat,
                            float* dw_part, int n_split, cudaStream_t s) {
  if (g.Ld <= 64) return rout_bwd_lm<T, 64>(g, drow, lat, w_rout, dlat, dw_part, n_split, s);
  return rout_bwd_lm<T, 128>(g, drow, lat, w_rout, dlat, dw_part, n_split, s);
}

#define INST(T)                                                                                          \
  template cudaError_t launch_gate_fwd<T>(const Geom&, const T*, const T*, const T*, const float*,        \
                                          const float*, const float*, T*, cudaStream_t);                  \
  template cudaError_t launch_gate_bwd<T>(const Geom&, const T*, const T*, const T*, const float*,        \
                                          const float*, const float*, const T*, T*, float*, float*,       \
                                          float*, int, cudaStream_t);                                     \
  template cudaError_t launch_rout_bwd<T>(const Geom&, const float*, const T*, const T*, float*, float*,  \
                                          int, cudaStream_t);
INST(float)
INST(bf16)
#undef INST

}  // namespace llattn
