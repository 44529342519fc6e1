// K1: latent-memory pooling of x (models.py:159-230).
//
// Chunk mode (models.py:159-214): pooled[b,c] = mean of x[b, c*cs : min((c+1)*cs, T)]
// over the true token count. Query-block mode (models.py:216-230): mean over
// bs tokens with zero padding counted (divisor bs even for the ragged block).
//
// HBM-bound: every element of x is read once, the pooled rows written once.
// One thread owns 16 bytes of a row (8 bf16 / 4 fp32 columns) and walks the
// chunk's tokens; consecutive threads own consecutive 16-byte columns, so each
// token row is read fully coalesced. Accumulation is fp32.
#include "common.cuh"

namespace llattn {
namespace {

template <typename T, int V>
struct Vec;
template <>
struct Vec<bf16, 8> {
  __device__ static void load(const bf16* p, float* o) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(bf16* p, const float* o) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec<float, 4> {
  __device__ static void load(const float* p, float* o) {
    float4 u = *reinterpret_cast<const float4*>(p);
    o[0] = u.x; o[1] = u.y; o[2] = u.z; o[3] = u.w;
  }
  __device__ static void store(float* p, const float* o) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
  }
};
template <typename T>
struct Vec<T, 1> {
  __device__ static void load(const T* p, float* o) { o[0] = to_f<T>(*p); }
  __device__ static void store(T* p, const float* o) { *p = from_f<T>(o[0]); }
};

// rows of size `size`; row r covers tokens [r*size, min((r+1)*size, T)).
// divisor: true count (chunks) or `size` (query blocks).
template <typename T, int V>
__global__ void __launch_bounds__(256) pool_fwd_kernel(const T* __restrict__ x, T* __restrict__ out,
                                                       int T_, int64_t d, int rows, int size,
                                                       int full_divisor) {
  const int b = blockIdx.z, r = blockIdx.y;
  const int64_t col = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * V;
  if (col >= d) return;
  const int t0 = r * size;
  const int t1 = min(t0 + size, T_);
  const T* src = x + ((int64_t)b * T_ + t0) * d + col;
  float acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;
  int t = t0;
  // four independent rows in flight per iteration
  for (; t + 4 <= t1; t += 4) {
    float v0[V], v1[V], v2[V], v3[V];
    Vec<T, V>::load(src, v0);
    Vec<T, V>::load(src + d, v1);
    Vec<T, V>::load(src + 2 * d, v2);
    Vec<T, V>::load(src + 3 * d, v3);
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] += (v0[i] + v1[i]) + (v2[i] + v3[i]);
    src += 4 * d;
  }
  for (; t < t1; ++t) {
    float v0[V];
    Vec<T, V>::load(src, v0);
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] += v0[i];
    src += d;
  }
  const float inv = 1.f / (float)(full_divisor ? size : (t1 - t0));
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] *= inv;
  Vec<T, V>::store(out + ((int64_t)b * rows + r) * d + col, acc);
}

// dx[b,t] = dout[b, t/size] / divisor(t/size): the mean's gradient spread over
// the row's tokens (models.py:195-199 / :223 through autograd).
template <typename T, int V>
__global__ void __launch_bounds__(256) pool_bwd_kernel(const T* __restrict__ dout, T* __restrict__ dx,
                                                       int T_, int64_t d, int rows, int size,
                                                       int full_divisor) {
  const int b = blockIdx.z, t = blockIdx.y;
  const int64_t col = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * V;
  if (col >= d) return;
  const int r = t / size;
  const int cnt = full_divisor ? size : (min((r + 1) * size, T_) - r * size);
  float v[V];
  Vec<T, V>::load(dout + ((int64_t)b * rows + r) * d + col, v);
  const float inv = 1.f / (float)cnt;
#pragma unroll
  for (int i = 0; i < V; ++i) v[i] *= inv;
  Vec<T, V>::store(dx + ((int64_t)b * T_ + t) * d + col, v);
}

template <typename T>
constexpr int vec_width() { return 16 / (int)sizeof(T); }

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

template <typename T>
cudaError_t launch_pool_fwd(const Geom& g, int mode, const T* x, T* out, int64_t d, cudaStream_t s) {
  const bool chunks = mode == LLATTN_POOL_CHUNKS;
  const int rows = chunks ? g.Nc : g.Tq;
  const int size = chunks ? g.cs : g.qbs;
  constexpr int V = vec_width<T>();
  if (d % V == 0 && aligned16(x) && aligned16(out)) {
    dim3 grid((unsigned)cdiv((int)(d / V), 256), rows, g.B);
    pool_fwd_kernel<T, V><<<grid, 256, 0, s>>>(x, out, g.T, d, rows, size, chunks ? 0 : 1);
  } else {
    dim3 grid((unsigned)cdiv((int)d, 256), rows, g.B);
    pool_fwd_kernel<T, 1><<<grid, 256, 0, s>>>(x, out, g.T, d, rows, size, chunks ? 0 : 1);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_pool_bwd(const Geom& g, int mode, const T* dout, T* dx, int64_t d, cudaStream_t s) {
  const bool chunks = mode == LLATTN_POOL_CHUNKS;
  const int rows = chunks ? g.Nc : g.Tq;
  const int size = chunks ? g.cs : g.qbs;
  constexpr int V = vec_width<T>();
  if (d % V == 0 && aligned16(dout) && aligned16(dx)) {
    dim3 grid((unsigned)cdiv((int)(d / V), 256), g.T, g.B);
    pool_bwd_kernel<T, V><<<grid, 256, 0, s>>>(dout, dx, g.T, d, rows, size, chunks ? 0 : 1);
  } else {
    dim3 grid((unsigned)cdiv((int)d, 256), g.T, g.B);
    pool_bwd_kernel<T, 1><<<grid, 256, 0, s>>>(dout, dx, g.T, d, rows, size, chunks ? 0 : 1);
  }
  return cudaGetLastError();
}

template cudaError_t launch_pool_fwd<float>(const Geom&, int, const float*, float*, int64_t, cudaStream_t);
template cudaError_t launch_pool_fwd<bf16>(const Geom&, int, const bf16*, bf16*, int64_t, cudaStream_t);
template cudaError_t launch_pool_bwd<float>(const Geom&, int, const float*, float*, int64_t, cudaStream_t);
template cudaError_t launch_pool_bwd<bf16>(const Geom&, int, const bf16*, bf16*, int64_t, cudaStream_t);

}  // namespace llattn
