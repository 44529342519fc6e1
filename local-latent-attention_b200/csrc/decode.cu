// One decode step of the attention core: the output row of the newest token
// t = T-1 of a T-token prefix, from a cache of the prefix's qkv rows. It is
// the last row of the full forward of that prefix (models.py:307-462 with
// every size derived from T, as the reference's generation loop recomputes
// it, generate.py:188-202), without recomputing the other T-1 rows.
//
// One CTA per (head h, sequence b), 4 warps, fp32 arithmetic (key rows are
// read whole by a warp, so every cache load is coalesced):
//   local  = softmax over keys [lo(t), t-1] of q_t.k_j / sqrt(hd), times v
//            (window and block-boundary mask of models.py:245-292), rounded
//            to the activation dtype as the forward stores local_out
//   lat    = causal-chunk softmax of rq.gk (chunks j < qid(t)) times gv,
//            rounded like the forward's lat (models.py:361-375)
//   remote = lat W_rout[h]^T + b_rout[h]                  (models.py:392-414)
//   w      = sigmoid(local.g_l + gate_bias - remote.g_r); mixed = w local +
//            (1 - w) remote                               (models.py:417-438)
// The work per token is a few hundred KB of cache reads: latency-bound
// vector work, no tensor-core tile to fill.
#include <math.h>

#include "common.cuh"

namespace llattn {
namespace {

constexpr int kDecThreads = 128;

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < kDecThreads / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < kDecThreads / 32; ++i) r += red[i];
  return r;
}

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f<T>(from_f<T>(v));
}

// smem: scores [max(min(W, T), Nc)] fp32, q [hd], lat [Ld], local [hd],
// remote [hd], red [32], P V partials [4][hd]
template <typename T>
__global__ void __launch_bounds__(kDecThreads) decode_kernel(Geom g, int64_t cache_stride_b, const T* __restrict__ qkv,
                                                             const T* __restrict__ rq_row, const T* __restrict__ gkv,
                                                             const T* __restrict__ w_rout,
                                                             const float* __restrict__ b_rout,
                                                             const float* __restrict__ g_local,
                                                             const float* __restrict__ g_remote, T* __restrict__ out,
                                                             int score_cap) {
  extern __shared__ float dec_smem[];
  float* sc = dec_smem;
  float* q = sc + score_cap;
  float* lat = q + g.hd;
  float* loc = lat + g.Ld;
  float* rem = loc + g.hd;
  float* red = rem + g.hd;
  float* part = red + 32;  // [kDecThreads / 32][hd] P V partials
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int t = g.T - 1;
  const int64_t row3 = (int64_t)3 * g.d;  // elements per cached token row
  const T* base = qkv + (int64_t)b * cache_stride_b;

  // ---- local branch: each warp takes every 4th key; a key's row is read by
  // the whole warp (lane l: columns l, l+32, ...), so every load is coalesced
  const float qs = g.scale * 1.4426950408889634f;  // scores in log2 units
  for (int c = tid; c < g.hd; c += kDecThreads) q[c] = to_f<T>(base[(int64_t)t * row3 + h * g.hd + c]) * qs;
  __syncthreads();
  const int lo = local_lo(g, t), nk = t - lo;  // keys lo .. t-1
  const int warp = tid / 32, lane = tid % 32;
  constexpr int NW = kDecThreads / 32;
  float mx = -INFINITY;
#pragma unroll 2
  for (int i = warp; i < nk; i += NW) {
    const T* k = base + (int64_t)(lo + i) * row3 + g.d + h * g.hd;
    float s = 0.f;
    for (int c = lane; c < g.hd; c += 32) s = fmaf(q[c], to_f<T>(k[c]), s);
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) sc[i] = s;
    mx = fmaxf(mx, s);
  }
  mx = block_max(mx, red);  // its barriers also publish the sc writes
  float l = 0.f;
  for (int i = tid; i < nk; i += kDecThreads) {
    const float p = exp2f(sc[i] - mx);
    sc[i] = p;
    l += p;
  }
  l = block_sum(l, red);
  const float inv = nk > 0 ? 1.f / l : 0.f;
  // P V: per-warp partial sums over its keys (lane: columns lane + 32u),
  // then the NW partials summed per column through shared memory
  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // hd <= 128
#pragma unroll 2
  for (int i = warp; i < nk; i += NW) {
    const float p = sc[i];
    const T* v = base + (int64_t)(lo + i) * row3 + 2 * g.d + h * g.hd;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (lane + 32 * u < g.hd) acc[u] = fmaf(p, to_f<T>(v[lane + 32 * u]), acc[u]);
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (lane + 32 * u < g.hd) part[warp * g.hd + lane + 32 * u] = acc[u];
  __syncthreads();
  for (int c = tid; c < g.hd; c += kDecThreads) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) a += part[w * g.hd + c];
    loc[c] = round_to<T>(a * inv);
  }
  __syncthreads();

  // ---- latent branch: row r = t / qbs sees chunks j < qid(r)
  const int qid = row_qid(g, t / g.qbs);
  const T* rqb = rq_row + (int64_t)b * g.Ld;
  const T* gkb = gkv + (int64_t)b * g.Nc * 2 * g.Ld;
  for (int lh = 0; lh < g.Lh; ++lh) {
    float lm = -INFINITY;
    for (int j = tid; j < qid; j += kDecThreads) {
      const T* k = gkb + (int64_t)j * 2 * g.Ld + lh * g.ldh;
      float s = 0.f;
      for (int e = 0; e < g.ldh; ++e) s = fmaf(to_f<T>(rqb[lh * g.ldh + e]), to_f<T>(k[e]), s);
      s *= g.lat_scale;
      sc[j] = s;
      lm = fmaxf(lm, s);
    }
    lm = block_max(lm, red);
    float ll = 0.f;
    for (int j = tid; j < qid; j += kDecThreads) {
      const float p = expf(sc[j] - lm);
      sc[j] = p;
      ll += p;
    }
    ll = block_sum(ll, red);
    const float linv = qid > 0 ? 1.f / ll : 0.f;
    for (int e = tid; e < g.ldh; e += kDecThreads) {
      float a = 0.f;
      for (int j = 0; j < qid; ++j) a = fmaf(sc[j], to_f<T>(gkb[(int64_t)j * 2 * g.Ld + g.Ld + lh * g.ldh + e]), a);
      lat[lh * g.ldh + e] = round_to<T>(a * linv);
    }
    __syncthreads();
  }

  // ---- remote row of head h, gate, mix
  float sl = 0.f, sr = 0.f;
  for (int c = tid; c < g.hd; c += kDecThreads) {
    const int col = h * g.hd + c;
    const T* wr = w_rout + (int64_t)col * g.Ld;
    float r = 0.f;
    for (int e = 0; e < g.Ld; ++e) r = fmaf(lat[e], to_f<T>(wr[e]), r);
    r += b_rout[col];
    rem[c] = r;
    sl = fmaf(loc[c], g_local[c], sl);
    sr = fmaf(r, g_remote[c], sr);
  }
  sl = block_sum(sl, red);
  sr = block_sum(sr, red);
  const float x = sl + g.gate_bias - sr;
  const float wl = 1.f / (1.f + expf(-x)), wr = 1.f / (1.f + expf(x));
  for (int c = tid; c < g.hd; c += kDecThreads)
    out[(int64_t)b * g.d + h * g.hd + c] = from_f<T>(wl * loc[c] + wr * rem[c]);
}

}  // namespace

template <typename T>
cudaError_t launch_decode(const Geom& g, int64_t cache_len, const T* qkv, const T* rq_row, const T* gkv,
                          const T* w_rout, const float* b_rout, const float* g_local, const float* g_remote, T* out,
                          cudaStream_t s) {
  const int nk_max = g.W < g.T ? g.W : g.T;  // keys of the newest row: at most min(W, t)
  const int cap = nk_max > g.Nc ? nk_max : g.Nc;
  const size_t smem = sizeof(float) * ((size_t)cap + (3 + kDecThreads / 32) * g.hd + g.Ld + 32);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = set_smem_once(decode_kernel<T>, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(g.H, g.B);
  decode_kernel<T><<<grid, kDecThreads, smem, s>>>(g, cache_len * 3 * g.d, qkv, rq_row, gkv, w_rout, b_rout, g_local,
                                                  g_remote, out, cap);
  return cudaGetLastError();
}

template cudaError_t launch_decode<float>(const Geom&, int64_t, const float*, const float*, const float*, const float*,
                                          const float*, const float*, const float*, float*, cudaStream_t);
template cudaError_t launch_decode<bf16>(const Geom&, int64_t, const bf16*, const bf16*, const bf16*, const bf16*,
                                         const float*, const float*, const float*, bf16*, cudaStream_t);

}  // namespace llattn
