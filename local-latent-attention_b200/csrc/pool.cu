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
#include <algorithm>

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
// With accumulate set, dx += that instead (one read-modify-write of dx, so
// the other gradient contributions to x need no separate add).
template <typename T, int V>
__global__ void __launch_bounds__(256) pool_bwd_kernel(const T* __restrict__ dout, T* __restrict__ dx,
                                                       int T_, int64_t d, int rows, int size,
                                                       int full_divisor, int accumulate) {
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
  T* dst = dx + ((int64_t)b * T_ + t) * d + col;
  if (accumulate) {
    float o[V];
    Vec<T, V>::load(dst, o);
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] += o[i];
  }
  Vec<T, V>::store(dst, v);
}

// Pooling fused with the latent projections (llattn_pool_proj_*). The
// pooled means are linear, so chunk_mean(x) W^T + b = chunk_mean(x W^T) + b
// and the same for the query-block means (models.py:159-230, :333-347): the
// projections run per token as ONE GEMM z = x [W_rkv; W_rq]^T ([B*T, 3Ld],
// no bias), and these kernels pool the 3Ld-wide rows of z instead of the
// d-wide rows of x. Part 0 = gkv (columns [0, 2Ld) of z, chunk means over
// the true count, + b_rkv), part 1 = rq (columns [2Ld, 3Ld), query-block
// means with zero padding counted, or the token's own row when qbs = 1,
// + b_rq). Thread = one (output row, 16-byte column group) item.
// Block layout: the part's ng = cols / V column groups (ng <= 256) x slots =
// 256 / ng thread slots; `split` slots share one output row's tokens (token
// t0 + k*split + sub for slot sub) and are summed in shared memory in a fixed
// order, rpb = slots / split output rows per block.
struct PoolPart {
  int col0, cols, rows, size, full_divisor, split, rpb, blocks;
};

template <typename T, int V>
__global__ void __launch_bounds__(256) pool_proj_fwd_kernel(const T* __restrict__ z, int ldz, int T_, int B,
                                                            PoolPart p0, PoolPart p1, const T* __restrict__ b0,
                                                            const T* __restrict__ b1, T* __restrict__ out0,
                                                            T* __restrict__ out1) {
  __shared__ float red[256 * V];
  const PoolPart p = blockIdx.y ? p1 : p0;
  if ((int)blockIdx.x >= p.blocks) return;
  const T* bias = blockIdx.y ? b1 : b0;
  T* out = blockIdx.y ? out1 : out0;
  const int ng = p.cols / V;
  const int cg = threadIdx.x % ng, slot = threadIdx.x / ng;
  const int slots = 256 / ng;
  const int rr = slot / p.split, sub = slot % p.split;
  const int br = blockIdx.x * p.rpb + rr;  // b * rows + r
  const bool live = slot < slots && rr < p.rpb && br < B * p.rows;
  float acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;
  int t0 = 0, t1 = 0;
  if (live) {
    const int b = br / p.rows, r = br % p.rows;
    t0 = r * p.size;
    t1 = min(t0 + p.size, T_);
    const T* src = z + ((size_t)b * T_ + t0 + sub) * ldz + p.col0 + cg * V;
    const size_t step = (size_t)p.split * ldz;
    int t = t0 + sub;
    for (; t + 3 * p.split < t1; t += 4 * p.split) {  // four rows in flight
      float v0[V], v1[V], v2[V], v3[V];
      Vec<T, V>::load(src, v0);
      Vec<T, V>::load(src + step, v1);
      Vec<T, V>::load(src + 2 * step, v2);
      Vec<T, V>::load(src + 3 * step, v3);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += (v0[i] + v1[i]) + (v2[i] + v3[i]);
      src += 4 * step;
    }
    for (; t < t1; t += p.split) {
      float v0[V];
      Vec<T, V>::load(src, v0);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += v0[i];
      src += step;
    }
  }
  if (p.split > 1) {
#pragma unroll
    for (int i = 0; i < V; ++i) red[threadIdx.x * V + i] = acc[i];
    __syncthreads();
    if (!live || sub != 0) return;
    for (int k = 1; k < p.split; ++k) {
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += red[(threadIdx.x + k * ng) * V + i];
    }
  } else if (!live) {
    return;
  }
  const float inv = 1.f / (float)(p.full_divisor ? p.size : (t1 - t0));
  float bv[V];
  if (bias) {
    Vec<T, V>::load(bias + cg * V, bv);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) bv[i] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = fmaf(acc[i], inv, bv[i]);
  Vec<T, V>::store(out + (size_t)br * p.cols + cg * V, acc);
}

// The gradient of the above with respect to z: dz[b*T + t, col0 + j] =
// dout[b, row(t), j] / divisor(row(t)); thread = one (token, column group),
// 32-bit indexing (the host checks B*T*ng < 2^31).
template <typename T, int V>
__global__ void __launch_bounds__(256) pool_proj_bwd_kernel(const T* __restrict__ d0, const T* __restrict__ d1,
                                                            T* __restrict__ dz, int ldz, int T_, int B,
                                                            PoolPart p0, PoolPart p1) {
  const PoolPart p = blockIdx.y ? p1 : p0;
  const T* dout = blockIdx.y ? d1 : d0;
  const unsigned ng = (unsigned)(p.cols / V);
  const unsigned item = blockIdx.x * blockDim.x + threadIdx.x;
  if (item >= (unsigned)B * (unsigned)T_ * ng) return;
  const unsigned cg = item % ng, bt = item / ng;
  const unsigned b = bt / (unsigned)T_, t = bt % (unsigned)T_;
  const int r = (int)t / p.size;
  const int cnt = p.full_divisor ? p.size : (min((r + 1) * p.size, T_) - r * p.size);
  float v[V];
  Vec<T, V>::load(dout + ((size_t)b * p.rows + r) * p.cols + cg * V, v);
  const float inv = 1.f / (float)cnt;
#pragma unroll
  for (int i = 0; i < V; ++i) v[i] *= inv;
  Vec<T, V>::store(dz + (size_t)bt * ldz + p.col0 + cg * V, v);
}

// Column sums of a row-major [rows, cols] matrix (the bias gradient of a
// linear layer: the sum of its output gradient over tokens), fp32
// accumulation. Block: 32 column groups of V columns x 8 row lanes; blockIdx.y
// takes a contiguous row range and writes its fp32 partial row to part[y].
template <typename T, int V>
__global__ void __launch_bounds__(256) colsum_part_kernel(const T* __restrict__ g, int64_t rows, int64_t cols,
                                                          int64_t ld, int64_t rows_per_split,
                                                          float* __restrict__ part) {
  __shared__ float red[8][32 * V + 1];
  const int cg = threadIdx.x & 31, rl = threadIdx.x >> 5;
  const int64_t col = ((int64_t)blockIdx.x * 32 + cg) * V;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_split;
  const int64_t r1 = min(rows, r0 + rows_per_split);
  float acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;
  if (col < cols) {
    int64_t r = r0 + rl;
    for (; r + 56 < r1; r += 64) {  // eight rows in flight per thread
      float v[8][V];
#pragma unroll
      for (int k = 0; k < 8; ++k) Vec<T, V>::load(g + (r + 8 * k) * ld + col, v[k]);
#pragma unroll
      for (int i = 0; i < V; ++i)
        acc[i] += ((v[0][i] + v[1][i]) + (v[2][i] + v[3][i])) + ((v[4][i] + v[5][i]) + (v[6][i] + v[7][i]));
    }
    for (; r + 24 < r1; r += 32) {
      float v0[V], v1[V], v2[V], v3[V];
      Vec<T, V>::load(g + r * ld + col, v0);
      Vec<T, V>::load(g + (r + 8) * ld + col, v1);
      Vec<T, V>::load(g + (r + 16) * ld + col, v2);
      Vec<T, V>::load(g + (r + 24) * ld + col, v3);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += (v0[i] + v1[i]) + (v2[i] + v3[i]);
    }
    for (; r < r1; r += 8) {
      float v0[V];
      Vec<T, V>::load(g + r * ld + col, v0);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += v0[i];
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) red[rl][cg * V + i] = acc[i];
  __syncthreads();
  // 256 threads sum the 8 row lanes of the block's 32 * V columns
  for (int c = threadIdx.x; c < 32 * V; c += 256) {
    const int64_t oc = (int64_t)blockIdx.x * 32 * V + c;
    if (oc < cols) {
      float s = red[0][c];
#pragma unroll
      for (int k = 1; k < 8; ++k) s += red[k][c];
      part[(int64_t)blockIdx.y * cols + oc] = s;
    }
  }
}

template <typename T>
constexpr int vec_width() { return 16 / (int)sizeof(T); }

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// threads per block for n column groups: up to 256, no idle warps when n < 256
inline int col_threads(int64_t n) { return n >= 256 ? 256 : (int)((n + 31) / 32 * 32); }

}  // namespace

template <typename T>
cudaError_t launch_pool_fwd(const Geom& g, int mode, const T* x, T* out, int64_t d, cudaStream_t s) {
  const bool chunks = mode == LLATTN_POOL_CHUNKS;
  const int rows = chunks ? g.Nc : g.Tq;
  const int size = chunks ? g.cs : g.qbs;
  constexpr int V = vec_width<T>();
  if (d % V == 0 && aligned16(x) && aligned16(out)) {
    const int nt = col_threads(d / V);
    dim3 grid((unsigned)cdiv((int)(d / V), nt), rows, g.B);
    pool_fwd_kernel<T, V><<<grid, nt, 0, s>>>(x, out, g.T, d, rows, size, chunks ? 0 : 1);
  } else {
    const int nt = col_threads(d);
    dim3 grid((unsigned)cdiv((int)d, nt), rows, g.B);
    pool_fwd_kernel<T, 1><<<grid, nt, 0, s>>>(x, out, g.T, d, rows, size, chunks ? 0 : 1);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_pool_bwd(const Geom& g, int mode, const T* dout, T* dx, int64_t d, int accumulate,
                            cudaStream_t s) {
  const bool chunks = mode == LLATTN_POOL_CHUNKS;
  const int rows = chunks ? g.Nc : g.Tq;
  const int size = chunks ? g.cs : g.qbs;
  constexpr int V = vec_width<T>();
  if (d % V == 0 && aligned16(dout) && aligned16(dx)) {
    const int nt = col_threads(d / V);
    dim3 grid((unsigned)cdiv((int)(d / V), nt), g.T, g.B);
    pool_bwd_kernel<T, V><<<grid, nt, 0, s>>>(dout, dx, g.T, d, rows, size, chunks ? 0 : 1, accumulate);
  } else {
    const int nt = col_threads(d);
    dim3 grid((unsigned)cdiv((int)d, nt), g.T, g.B);
    pool_bwd_kernel<T, 1><<<grid, nt, 0, s>>>(dout, dx, g.T, d, rows, size, chunks ? 0 : 1, accumulate);
  }
  return cudaGetLastError();
}

namespace {
// column groups of v elements; split / rows per block as described at the kernel
PoolPart pool_part(int col0, int cols, int rows, int size, int full_divisor, int v, int B) {
  PoolPart p{col0, cols, rows, size, full_divisor, 1, 1, 0};
  const int slots = 256 / (cols / v);
  int split = 1;
  while (split * 2 <= slots && split * 2 <= size) split *= 2;
  p.split = split;
  p.rpb = slots / split;
  p.blocks = cdiv(B * rows, p.rpb);
  return p;
}
}  // namespace

template <typename T>
cudaError_t launch_pool_proj_fwd(const Geom& g, const T* z, int64_t ldz, const T* b_rkv, const T* b_rq, T* gkv,
                                 T* rq, cudaStream_t s) {
  constexpr int V = vec_width<T>();
  const bool vec = g.Ld % V == 0 && ldz % V == 0 && aligned16(z) && aligned16(gkv) && aligned16(rq) &&
                   (!b_rkv || aligned16(b_rkv)) && (!b_rq || aligned16(b_rq));
  const int v = vec ? V : 1;
  if (2 * g.Ld / v > 256 || ldz > INT32_MAX || (int64_t)g.B * g.T * ldz >= ((int64_t)1 << 40))
    return cudaErrorInvalidValue;
  const PoolPart p0 = pool_part(0, 2 * g.Ld, g.Nc, g.cs, 0, v, g.B);
  const PoolPart p1 = pool_part(2 * g.Ld, g.Ld, g.Tq, g.qbs, 1, v, g.B);
  dim3 grid((unsigned)std::max(p0.blocks, p1.blocks), 2);
  if (vec)
    pool_proj_fwd_kernel<T, V><<<grid, 256, 0, s>>>(z, (int)ldz, g.T, g.B, p0, p1, b_rkv, b_rq, gkv, rq);
  else
    pool_proj_fwd_kernel<T, 1><<<grid, 256, 0, s>>>(z, (int)ldz, g.T, g.B, p0, p1, b_rkv, b_rq, gkv, rq);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_pool_proj_bwd(const Geom& g, const T* dgkv, const T* drq, T* dz, int64_t ldz, cudaStream_t s) {
  constexpr int V = vec_width<T>();
  const bool vec = g.Ld % V == 0 && ldz % V == 0 && aligned16(dz) && aligned16(dgkv) && aligned16(drq);
  const int v = vec ? V : 1;
  const int64_t items = (int64_t)g.B * g.T * (2 * g.Ld / v);  // part 0 is the wider one
  if (items >= ((int64_t)1 << 31) || ldz > INT32_MAX) return cudaErrorInvalidValue;
  const PoolPart p0{0, 2 * g.Ld, g.Nc, g.cs, 0, 1, 1, 0};
  const PoolPart p1{2 * g.Ld, g.Ld, g.Tq, g.qbs, 1, 1, 1, 0};
  dim3 grid((unsigned)((items + 255) / 256), 2);
  if (vec)
    pool_proj_bwd_kernel<T, V><<<grid, 256, 0, s>>>(dgkv, drq, dz, (int)ldz, g.T, g.B, p0, p1);
  else
    pool_proj_bwd_kernel<T, 1><<<grid, 256, 0, s>>>(dgkv, drq, dz, (int)ldz, g.T, g.B, p0, p1);
  return cudaGetLastError();
}

template cudaError_t launch_pool_proj_fwd<float>(const Geom&, const float*, int64_t, const float*, const float*,
                                                 float*, float*, cudaStream_t);
template cudaError_t launch_pool_proj_fwd<bf16>(const Geom&, const bf16*, int64_t, const bf16*, const bf16*, bf16*,
                                                bf16*, cudaStream_t);
template cudaError_t launch_pool_proj_bwd<float>(const Geom&, const float*, const float*, float*, int64_t,
                                                 cudaStream_t);
template cudaError_t launch_pool_proj_bwd<bf16>(const Geom&, const bf16*, const bf16*, bf16*, int64_t,
                                                cudaStream_t);

// SMs of the current device, cached per device
int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 148;
  }
  return cache[dev];
}

int colsum_splits(int64_t rows, int64_t cols, int elem_bytes) {
  const int64_t v = 16 / elem_bytes;
  const int64_t gx = (cols + 32 * v - 1) / (32 * v);
  // at most 8 blocks per SM (the launch takes what fits resident), at least
  // 64 rows per block
  int64_t splits = (148 * 8 + gx - 1) / gx;
  splits = std::min<int64_t>(splits, (rows + 63) / 64);
  return (int)std::max<int64_t>(splits, 1);
}

template <typename K>
int colsum_occupancy(K kernel) {
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, 256, 0) != cudaSuccess || occ < 1) return 1;
  return occ;
}

template <typename T, typename To>
cudaError_t launch_colsum(const T* g, int64_t rows, int64_t cols, float* part, To* out, cudaStream_t s, int64_t ld) {
  constexpr int V = vec_width<T>();
  if (ld <= 0) ld = cols;
  const bool vec = cols % V == 0 && ld % V == 0 && aligned16(g);
  const int gx = vec ? cdiv((int)(cols / V), 32) : cdiv((int)cols, 32);
  // one wave: as many row splits as fit resident beside the column groups
  static const int occ_v = colsum_occupancy(colsum_part_kernel<T, V>);
  static const int occ_1 = colsum_occupancy(colsum_part_kernel<T, 1>);
  const int occ = vec ? occ_v : occ_1, sms = sm_count();
  const int splits = std::max(1, std::min(colsum_splits(rows, cols, (int)sizeof(T)), sms * occ / gx));
  const int64_t per = (rows + splits - 1) / splits;
  if (vec)
    colsum_part_kernel<T, V><<<dim3(gx, splits), 256, 0, s>>>(g, rows, cols, ld, per, part);
  else
    colsum_part_kernel<T, 1><<<dim3(gx, splits), 256, 0, s>>>(g, rows, cols, ld, per, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_reduce_parts<To>(part, splits, cols, out, s);
}

template cudaError_t launch_colsum<float, float>(const float*, int64_t, int64_t, float*, float*, cudaStream_t, int64_t);
template cudaError_t launch_colsum<bf16, bf16>(const bf16*, int64_t, int64_t, float*, bf16*, cudaStream_t, int64_t);
template cudaError_t launch_colsum<bf16, float>(const bf16*, int64_t, int64_t, float*, float*, cudaStream_t, int64_t);
template cudaError_t launch_pool_fwd<float>(const Geom&, int, const float*, float*, int64_t, cudaStream_t);
template cudaError_t launch_pool_fwd<bf16>(const Geom&, int, const bf16*, bf16*, int64_t, cudaStream_t);
template cudaError_t launch_pool_bwd<float>(const Geom&, int, const float*, float*, int64_t, int, cudaStream_t);
template cudaError_t launch_pool_bwd<bf16>(const Geom&, int, const bf16*, bf16*, int64_t, int, cudaStream_t);

}  // namespace llattn
