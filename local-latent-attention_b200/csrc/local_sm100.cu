// Tensor-core (tcgen05 + TMA) kernels of the local branch and of the
// r_out / gate backward for bf16 activations on sm_100a, and their host-side
// launchers (tensor maps, shared-memory sizing). The kernels live in:
//   local_sm100_fwd_pp.cuh  forward, one 128-query tile per CTA and two CTAs
//                           per SM (two tiles per CTA with LLATTN_FWD_PAIR=1),
//                           fused remote projection + gate + mix epilogue
//   local_sm100_bwd.cuh     dq (units of query tiles) and dk/dv (units of key tiles), persistent
//   gate_sm100.cuh          gate / r_out backward and the dW_rout GEMM
//   latent_sm100.cuh        latent attention forward / backward (up to 512 chunks)
// Windowed causal mask of the reference (models.py:232-305): key j is
// visible from query t iff 0 < t-j <= W and j >= qs(t) - W + 1.
//
// Every wait is bounded (mbar_wait): on timeout a kernel records a fault
// bit in g_fault_word, tells its other warps to stop, waits for its own
// in-flight copies, frees its TMEM and returns; the host reads the word with
// llattn_fault_status().
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "sm100.cuh"
#include "sm100_ptx.cuh"

namespace llattn {
namespace sm100 {

// Nonzero once any tensor-core kernel gave up on a wait; every later wait
// (in any CTA) then returns at once, so a broken launch ends within about a
// second instead of timing out CTA by CTA.
__device__ unsigned int g_fault_word = 0;

#if defined(LLATTN_TRACE)
// diagnostic builds only: per-CTA phase timestamps (globaltimer, ns)
constexpr int kTraceCtas = 1024, kTraceEv = 64;
__device__ unsigned long long g_trace[kTraceCtas][kTraceEv];
// LLATTN_TRACE selects which kernel records (1 forward, 2 dK/dV, 3 gate backward)
#define LLATTN_TRACE_K(kid, ev)                                                                 \
  do {                                                                                          \
    if (LLATTN_TRACE == (kid)) {                                                                \
      const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);         \
      if (cta_ < kTraceCtas && (ev) < kTraceEv) g_trace[cta_][(ev)] = ptx::globaltimer_ns(); \
    }                                                                                           \
  } while (0)
#else
#define LLATTN_TRACE_K(kid, ev) \
  do {                          \
  } while (0)
#endif

namespace {

using namespace ptx;

constexpr int BM = 128;  // query rows per tile (= TMEM lanes)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum Fault : unsigned {
  kFaultProducer = 1u, kFaultMma = 2u, kFaultSoftmax = 4u, kFaultEpilogue = 8u,
};

// Records the fault in the device word (which stops every other wait at
// once), in the host-mapped word the entry points test before each launch
// (so the op fails loudly instead of returning abandoned outputs), and in
// this CTA's abort flag.
__device__ __forceinline__ void raise_fault(const Geom& g, unsigned bit, volatile int* abort) {
  atomicOr(&g_fault_word, bit);
  if (g.fault_host) {
    *g.fault_host |= bit;
    __threadfence_system();
  }
  if (abort) *abort = 1;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Sum of v[c] over the 32 lanes for column c = lane (recursive halving).
__device__ __forceinline__ float butterfly32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool up = lane & off;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = up ? v[i] : v[i + off];
      const float keep = up ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

#include "local_sm100_fwd_pp.cuh"
#include "local_sm100_bwd.cuh"
#include "gate_sm100.cuh"
#include "latent_sm100.cuh"
#include "gemm_sm100.cuh"

// ---------------------------------------------------------------------------
// host side

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Encoded tensor maps, cached by their full description (base address,
// sizes, strides, box, swizzle, L2 promotion): a training loop re-launches
// with the same buffers, and the maps are plain host data, so a hit skips
// the driver call. Direct-mapped, 1024 entries, under a mutex.
struct MapKey {
  const void* base;
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5];
  int rank, swz, l2;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};

CUresult encode_cached(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims,
                       const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz,
                       CUtensorMapL2promotion l2) {
  auto enc = get_encode();
  if (!enc) return CUDA_ERROR_NOT_SUPPORTED;
  MapKey k;
  std::memset(&k, 0, sizeof(k));
  k.base = base;
  for (int i = 0; i < rank; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
    if (i + 1 < rank) k.strides[i] = strides[i];
  }
  k.rank = rank;
  k.swz = (int)swz;
  k.l2 = (int)l2;
  uint64_t h = 1469598103934665603ull;  // FNV-1a over the key bytes
  const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
  for (size_t i = 0; i < sizeof(k); ++i) h = (h ^ p[i]) * 1099511628211ull;
  static std::mutex mu;
  static MapKey keys[1024];
  static CUtensorMap maps[1024];
  static bool used[1024];
  const int slot = (int)(h % 1024);
  std::lock_guard<std::mutex> lk(mu);
  if (used[slot] && keys[slot] == k) {
    *map = maps[slot];
    return CUDA_SUCCESS;
  }
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) {
    keys[slot] = k;
    maps[slot] = *map;
    used[slot] = true;
  }
  return r;
}

// [B, T, S, H, hd] bf16 viewed as 4-D (hd, S*H, T, B); box (64, 1, rows, 1).
// row_elems: elements between consecutive token rows (0 = slots_x_heads * hd)
bool make_rows_map(CUtensorMap* map, const void* base, int B, int T, int slots_x_heads, int hd, int rows = 128,
                   int64_t row_elems = 0) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t row = (cuuint64_t)(row_elems > 0 ? row_elems : (int64_t)slots_x_heads * hd) * 2;
  cuuint64_t dims[4] = {(cuuint64_t)hd, (cuuint64_t)slots_x_heads, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)hd * 2, row, (cuuint64_t)T * row};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_cached(map, 4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  return r == CUDA_SUCCESS;
}

// LLATTN_FORCE_SIMT=1 routes bf16 through the SIMT kernels (used by the tests
// to compare the two implementations of the same math).
// bf16 matrix [rows, cols] (cols contiguous) with box (64 cols, box_rows rows).
bool make_2d_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows = 64) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return encode_cached(map, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B) == CUDA_SUCCESS;
}

// bf16 matrix [rows, cols] with row stride ld elements, box (64 cols, box_rows rows).
bool make_ld_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return encode_cached(map, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B) == CUDA_SUCCESS;
}

// bf16 [B, T, d] as 3-D (d, T, B), box (64, 128, 1), 128-byte swizzle.
bool make_btd_map(CUtensorMap* map, const void* base, int B, int T, int d) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)T * d * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode_cached(map, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE) == CUDA_SUCCESS;
}


bool force_simt() {
  const char* e = std::getenv("LLATTN_FORCE_SIMT");
  return e && e[0] == '1';
}

template <int HD>
cudaError_t fwd_hd(const Geom& g, const void* qkv, void* local_out, float* lse, const GateEpilogue& ep,
                   cudaStream_t s) {
  CUtensorMap tq, tkv;
  if (!make_rows_map(&tq, qkv, g.B, g.T, 3 * g.H, g.hd, 128, g.ldq) ||
      !make_rows_map(&tkv, qkv, g.B, g.T, 3 * g.H, g.hd, 64, g.ldq))
    return cudaErrorInvalidValue;
  // two query tiles per CTA (ping-pong), one CTA per SM; the fused epilogue
  // stores local_out and mixed through 3-D maps (d, T, B) that clip at T
  CUtensorMap tlo, tmx, tlat, tw;
  if (!make_rows_map(&tlo, local_out, g.B, g.T, g.H, g.hd, 128) ||
      !make_rows_map(&tmx, ep.mixed ? ep.mixed : local_out, g.B, g.T, g.H, g.hd, 128))
    return cudaErrorInvalidValue;
  // remote-tile operands: lat rows [B, Tq, 64] (box 64 x 128 rows) and the
  // head's W_rout slice [d, 64] (box 64 x hd rows); unused without the fusion
  if (ep.lat) {
    if (!make_btd_map(&tlat, ep.lat, g.B, g.Tq, 64) || !make_2d_map(&tw, ep.w_rout, g.d, 64, HD))
      return cudaErrorInvalidValue;
  } else {
    tlat = tlo;
    tw = tlo;
  }
  // LLATTN_FWD_PAIR=1 selects the two-tiles-per-CTA variant (one CTA per SM)
  static const bool pair = [] {
    const char* e = std::getenv("LLATTN_FWD_PAIR");
    return e && e[0] == '1';
  }();
  if (pair) {
    const int smem = FwdPPLayout<HD, true>::BYTES;
    cudaError_t e = set_smem_once(local_fwd_pp_kernel<HD, true>, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(g.H, cdiv(g.T, 2 * BM), g.B);
    local_fwd_pp_kernel<HD, true><<<grid, FwdPPLayout<HD, true>::THREADS, smem, s>>>(
        tq, tkv, tlo, tmx, tlat, tw, g, static_cast<bf16*>(local_out), lse, ep);
  } else {
    const int smem = FwdPPLayout<HD, false>::BYTES;
    cudaError_t e = set_smem_once(local_fwd_pp_kernel<HD, false>, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(g.H, cdiv(g.T, BM), g.B);
    local_fwd_pp_kernel<HD, false><<<grid, FwdPPLayout<HD, false>::THREADS, smem, s>>>(
        tq, tkv, tlo, tmx, tlat, tw, g, static_cast<bf16*>(local_out), lse, ep);
  }
  return cudaGetLastError();
}

template <int HD>
cudaError_t dq_hd(const Geom& g, const void* qkv, const void* dl, const float* lse, const float* delta, void* dqkv,
                  cudaStream_t s) {
  CUtensorMap q128, q64, do128, st;
  if (!make_rows_map(&q128, qkv, g.B, g.T, 3 * g.H, g.hd, 128, g.ldq) ||
      !make_rows_map(&q64, qkv, g.B, g.T, 3 * g.H, g.hd, 64, g.ldq) ||
      !make_rows_map(&do128, dl, g.B, g.T, g.H, g.hd, 128) ||
      !make_rows_map(&st, dqkv, g.B, g.T, 3 * g.H, g.hd, 128, g.ldd))
    return cudaErrorInvalidValue;
  // persistent: one CTA per SM walks the (h, query tile, b) units
  const int smem = DqpLayout<HD>::BYTES;  // the kernel's shared memory is 1024-byte aligned
  cudaError_t e = set_smem_once(local_dq_persist_kernel<HD>, smem);
  if (e != cudaSuccess) return e;
  const int n_units = g.H * cdiv(g.T, BM) * g.B;
  local_dq_persist_kernel<HD><<<std::min(n_units, sm_count()), 320, smem, s>>>(q128, q64, do128, st, g, lse, delta,
                                                                               n_units);
  return cudaGetLastError();
}

template <int HD>
cudaError_t dkv_hd(const Geom& g, const void* qkv, const void* dl, const float* lse, const float* delta, void* dqkv,
                   cudaStream_t s) {
  CUtensorMap q128, q64, do64, st;
  if (!make_rows_map(&q128, qkv, g.B, g.T, 3 * g.H, g.hd, 128, g.ldq) ||
      !make_rows_map(&q64, qkv, g.B, g.T, 3 * g.H, g.hd, 64, g.ldq) ||
      !make_rows_map(&do64, dl, g.B, g.T, g.H, g.hd, 64) ||
      !make_rows_map(&st, dqkv, g.B, g.T, 3 * g.H, g.hd, 128, g.ldd))
    return cudaErrorInvalidValue;
  const int smem = DkvLayout<HD>::BYTES;  // the kernel's shared memory is 1024-byte aligned
  cudaError_t e = set_smem_once(local_dkv_tc_kernel<HD>, smem);
  if (e != cudaSuccess) return e;
  // persistent: one CTA per SM walks the (h, key tile, b) units
  const int n_units = g.H * cdiv(g.T, BM) * g.B;
  local_dkv_tc_kernel<HD><<<std::min(n_units, sm_count()), 320, smem, s>>>(q128, q64, do64, st, g, lse, delta, n_units);
  return cudaGetLastError();
}

template <int HD, int G>
cudaError_t gate_bwd_hd(const Geom& g, const GateBwd& a, cudaStream_t s) {
  CUtensorMap tlo, tdm, tdl, tdr;
  // per-head 4-D maps (hd, H, rows, B): a padded head_dim's extra columns
  // are zero-filled on load and clipped on store
  if (!make_rows_map(&tlo, a.local_out, 1, g.B * g.T, g.H, g.hd, 128) ||
      !make_rows_map(&tdm, a.dmixed, 1, g.B * g.T, g.H, g.hd, 128) ||
      !make_rows_map(&tdl, a.dl, g.B, g.T, g.H, g.hd, 128) || !make_rows_map(&tdr, a.dr, g.B, g.T, g.H, g.hd, 128))
    return cudaErrorInvalidValue;
  const int smem = GbLayout<HD, G>::BYTES + 1024;
  cudaError_t e = set_smem_once(gate_bwd_tc_kernel<HD, G>, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, BM), g.B);
  gate_bwd_tc_kernel<HD, G><<<grid, GbLayout<HD, G>::THREADS, smem, s>>>(
      tlo, tdm, tdl, tdr, g, static_cast<const bf16*>(a.lat), static_cast<const bf16*>(a.w_rout), a.b_rout, a.g_local,
      a.g_remote, a.delta, a.dlat_tok, a.dg_part);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(const Geom& g, int M, int N, int K, const void* A, int64_t lda, int a_mn, const void* B,
                        int64_t ldb, int b_mn, const GemmOut& o, int splits, cudaStream_t s) {
  if (M < 1 || N < 1 || K < 1 || splits < 1) return cudaErrorInvalidValue;
  if (((uintptr_t)A & 15) || ((uintptr_t)B & 15) || (lda % 8) || (ldb % 8)) return cudaErrorMisalignedAddress;
  CUtensorMap ta, tb;
  // K-major: [rows, K] tiles of 128 rows x 64 K; MN-major: [K, MN] panels of 64 MN x 64 K rows
  if (!(a_mn ? make_ld_map(&ta, A, K, M, lda, 64) : make_ld_map(&ta, A, M, K, lda, 128)) ||
      !(b_mn ? make_ld_map(&tb, B, K, N, ldb, 64) : make_ld_map(&tb, B, N, K, ldb, 128)))
    return cudaErrorInvalidValue;
  GemmArgs p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.k_per_split = cdiv(cdiv(K, splits), 64) * 64;
  p.bias = o.bias;
  p.C = o.C;
  p.ldc = o.ldc;
  p.c_bf16 = o.out_bf16;
  p.c_split = o.split_stride;
  p.rows_per_group = o.rows_per_group > 0 ? o.rows_per_group : M;
  p.group_stride = o.group_stride;
  p.row_step = o.row_step > 0 ? o.row_step : 1;
  p.colsum = o.colsum;
  p.colsum_split = o.colsum_split;
  const int smem = GemmLayout::BYTES + 1024;
  if (!o.colsum && splits == 1 && K > 0) {
    // persistent: two CTAs per SM walk the output tiles, double-buffered accumulators
    cudaError_t e = set_smem_once(gemm_tc_persistent_kernel, smem);
    if (e != cudaSuccess) return e;
    const int n_tiles = cdiv(N, 128) * cdiv(M, 128);
    gemm_tc_persistent_kernel<<<std::min(n_tiles, 2 * sm_count()), 192, smem, s>>>(ta, tb, g, p);
    return cudaGetLastError();
  }
  cudaError_t e = set_smem_once(gemm_tc_kernel, smem);
  if (e != cudaSuccess) return e;
  // every split runs (one whose K range is empty writes zeros): callers sum
  // exactly `splits` partials
  dim3 grid(cdiv(N, 128), cdiv(M, 128), splits);
  gemm_tc_kernel<<<grid, 192, smem, s>>>(ta, tb, g, p);
  return cudaGetLastError();
}

int gate_bwd_ctas(const Geom& g) { return g.B * cdiv(g.T, BM); }
int gate_dg_floats(const Geom& g) { return gate_dg_stride(g.hd, g.H); }

cudaError_t launch_gate_dgr_finalize(const Geom& g, const float* dg_sum, const void* w_rout, const float* b_rout,
                                     float* dg_remote, cudaStream_t s) {
  gate_dgr_finalize_kernel<<<cdiv(g.hd, 16), 256, 0, s>>>(g, dg_sum, static_cast<const bf16*>(w_rout), b_rout, dg_remote);
  return cudaGetLastError();
}

cudaError_t launch_gate_bwd(const Geom& g, const GateBwd& a, cudaStream_t s) {
  // one head group per CTA, two CTAs per SM, unless the heads' ds rows do not fit
  if (g.H <= gate_max_heads<1>()) {
    if (g.hd == 64) return gate_bwd_hd<64, 1>(g, a, s);
    return gate_bwd_hd<128, 1>(g, a, s);
  }
  if (g.hd == 64) return gate_bwd_hd<64, 2>(g, a, s);
  return gate_bwd_hd<128, 2>(g, a, s);
}

cudaError_t launch_rout_dw(const Geom& g, const void* dr, const void* lat, float* dw_part, float* db_part,
                           int n_split, cudaStream_t s) {
  CUtensorMap tm, tl;
  if (!make_2d_map(&tm, dr, (int64_t)g.B * g.T, g.d)) return cudaErrorInvalidValue;
  // token-wise queries: the lat rows of a 64-token chunk are one box of [B*Tq, 64]
  if (g.qbs == 1) {
    if (!make_2d_map(&tl, lat, (int64_t)g.B * g.Tq, 64, 64)) return cudaErrorInvalidValue;
  } else {
    tl = tm;
  }
  const int smem = DwLayout::BYTES + 1024;  // < 113 KB: two CTAs per SM
  cudaError_t e = set_smem_once(rout_dw_tc_kernel, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.d, 128), n_split);
  rout_dw_tc_kernel<<<grid, 192, smem, s>>>(tm, tl, g, static_cast<const bf16*>(lat), dw_part, db_part, n_split);
  return cudaGetLastError();
}

// latent head dim 32, or up to 64 as 64-wide tiles (ldh a multiple of 8,
// the columns past it zero); one 64-chunk key tile
bool latent_tc_ok(const Geom& g) {
  return !force_simt() && g.ldh <= 64 && g.ldh % 8 == 0 && g.Nc <= 64 && g.Tq >= 1;
}

int latent_tc_splits(const Geom& g) { return std::max(1, std::min(cdiv(g.Tq, BM), (2 * sm_count()) / (g.B * g.Lh))); }

cudaError_t launch_latent_bwd_tc(const Geom& g, const void* rq, const void* gkv, const float* lat_lse,
                                 const float* dlat, void* drq, float* part, int n_split, cudaStream_t s) {
  if (!latent_tc_ok(g)) return cudaErrorNotSupported;
  if (((uintptr_t)rq & 15) || ((uintptr_t)gkv & 15) || ((uintptr_t)dlat & 15) || ((uintptr_t)drq & 15))
    return cudaErrorMisalignedAddress;
  dim3 grid(n_split, g.Lh, g.B);
  auto run = [&](auto kern, int smem) -> cudaError_t {  // the kernel's shared memory is 1024-byte aligned
    cudaError_t e = set_smem_once(kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, 160, smem, s>>>(g, static_cast<const bf16*>(rq), static_cast<const bf16*>(gkv), lat_lse, dlat,
                                 static_cast<bf16*>(drq), part, n_split);
    return cudaGetLastError();
  };
  if (g.ldh <= 32) return run(latent_bwd_tc_kernel<32>, LatTcLayout<32>::BYTES);
  return run(latent_bwd_tc_kernel<64>, LatTcLayout<64>::BYTES);
}

// backward past one key tile: 64 < Nc <= 512 (the rows / keys kernel pair)
bool latent_tc_long_ok(const Geom& g) {
  return !force_simt() && g.ldh <= 64 && g.ldh % 8 == 0 && g.Nc > 64 && g.Nc <= 512 && g.Tq >= 1;
}

cudaError_t launch_latent_bwd_tc_long(const Geom& g, const void* rq, const void* gkv, const float* lat_lse,
                                      const float* dlat, void* drq, float* delta, float* part, int n_split_keys,
                                      cudaStream_t s) {
  if (!latent_tc_long_ok(g)) return cudaErrorNotSupported;
  if (((uintptr_t)rq & 15) || ((uintptr_t)gkv & 15) || ((uintptr_t)dlat & 15) || ((uintptr_t)drq & 15))
    return cudaErrorMisalignedAddress;
  const bf16* rq_ = static_cast<const bf16*>(rq);
  const bf16* gkv_ = static_cast<const bf16*>(gkv);
  // rows: 512 TMEM columns a CTA, so at least 116 KB of shared memory (one CTA per SM)
  {
    auto kern = g.ldh <= 32 ? latent_bwd_rows_tc_kernel<32> : latent_bwd_rows_tc_kernel<64>;
    const int cap = std::max(LatBwdRowsLayout::bytes(512), 116 * 1024);
    cudaError_t e = set_smem_once(kern, cap);
    if (e != cudaSuccess) return e;
    const int smem = std::max(LatBwdRowsLayout::bytes(g.Nc), 116 * 1024);
    const int n_split = std::max(1, std::min(cdiv(g.Tq, BM), (2 * sm_count()) / (g.B * g.Lh)));
    dim3 grid(n_split, g.Lh, g.B);
    kern<<<grid, 160, smem, s>>>(g, rq_, gkv_, lat_lse, dlat, static_cast<bf16*>(drq), delta, n_split);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  {
    auto kern = g.ldh <= 32 ? latent_bwd_keys_tc_kernel<32> : latent_bwd_keys_tc_kernel<64>;
    cudaError_t e = set_smem_once(kern, LatBwdKeysLayout::LAUNCH);
    if (e != cudaSuccess) return e;
    dim3 grid(cdiv(g.Nc, BM) * n_split_keys, g.Lh, g.B);
    kern<<<grid, 160, LatBwdKeysLayout::LAUNCH, s>>>(g, rq_, gkv_, lat_lse, dlat, delta, part, n_split_keys);
    return cudaGetLastError();
  }
}

// forward: up to 512 chunks (more than 64: the two-pass kernel over 64-key tiles)
bool latent_tc_fwd_ok(const Geom& g) {
  return !force_simt() && g.ldh <= 64 && g.ldh % 8 == 0 && g.Nc <= 512 && g.Tq >= 1;
}

cudaError_t launch_latent_fwd_tc(const Geom& g, const void* rq, const void* gkv, void* lat, float* lat_lse,
                                 cudaStream_t s) {
  if (!latent_tc_fwd_ok(g)) return cudaErrorNotSupported;
  if (((uintptr_t)rq & 15) || ((uintptr_t)gkv & 15) || ((uintptr_t)lat & 15)) return cudaErrorMisalignedAddress;
  if (g.Nc > 64) {
    auto kern = g.ldh <= 32 ? latent_fwd_tc_long_kernel<32> : latent_fwd_tc_long_kernel<64>;
    // the attribute covers the largest key set; a launch asks for at least
    // 80 KB so that no more than two CTAs (256 TMEM columns each) share an SM
    cudaError_t e = set_smem_once(kern, LatFwdLongLayout::bytes(512));
    if (e != cudaSuccess) return e;
    const int smem = std::max(LatFwdLongLayout::bytes(g.Nc), 80 * 1024);
    const int n_split = std::max(1, std::min(cdiv(g.Tq, BM), (2 * sm_count()) / (g.B * g.Lh)));
    dim3 grid(n_split, g.Lh, g.B);
    kern<<<grid, 160, smem, s>>>(g, static_cast<const bf16*>(rq), static_cast<const bf16*>(gkv),
                                 static_cast<bf16*>(lat), lat_lse, n_split);
    return cudaGetLastError();
  }
  const int smem = LatFwdTcLayout::BYTES;  // the kernel's shared memory is 1024-byte aligned
  auto kern = g.ldh <= 32 ? latent_fwd_tc_kernel<32> : latent_fwd_tc_kernel<64>;
  cudaError_t e = set_smem_once(kern, smem);
  if (e != cudaSuccess) return e;
  // up to four CTAs per SM (128 TMEM columns each)
  const int n_split = std::max(1, std::min(cdiv(g.Tq, BM), (4 * sm_count()) / (g.B * g.Lh)));
  dim3 grid(n_split, g.Lh, g.B);
  kern<<<grid, 160, smem, s>>>(g, static_cast<const bf16*>(rq), static_cast<const bf16*>(gkv),
                               static_cast<bf16*>(lat), lat_lse, n_split);
  return cudaGetLastError();
}

cudaError_t launch_dlat_rowsum(const Geom& g, const float* dlat_tok, float* dlat, cudaStream_t s) {
  const int64_t n = (int64_t)g.B * g.Tq * 64;
  dlat_rowsum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, dlat_tok, dlat);
  return cudaGetLastError();
}

bool fwd_supported(const Geom& g, int elt_bytes) {
  // head_dim 64, or 64 < hd <= 128 run as 128-wide tiles (the copies zero-fill
  // the columns past hd; 16-byte rows need hd % 8 == 0)
  const bool hd_ok = g.hd == 64 || (g.hd > 64 && g.hd <= 128 && g.hd % 8 == 0);
  return !force_simt() && elt_bytes == 2 && hd_ok && get_encode() != nullptr;
}

bool bwd_supported(const Geom& g, int elt_bytes) { return fwd_supported(g, elt_bytes); }

bool gate_fusable(const Geom& g) { return g.Ld == 64 && g.H <= kGateMaxHeads; }

cudaError_t launch_local_fwd(const Geom& g, const void* qkv, void* local_out, float* lse, const GateEpilogue& ep,
                             cudaStream_t s) {
  if (((uintptr_t)qkv & 15) || ((uintptr_t)local_out & 15)) return cudaErrorMisalignedAddress;
  if (ep.lat && (g.Ld != 64 || ((uintptr_t)ep.lat & 15) || ((uintptr_t)ep.w_rout & 15) ||
                 ((uintptr_t)ep.mixed & 15) || ((uintptr_t)ep.b_rout & 15) || ((uintptr_t)ep.g_local & 15) ||
                 ((uintptr_t)ep.g_remote & 15)))
    return cudaErrorMisalignedAddress;
  if (g.hd == 64) return fwd_hd<64>(g, qkv, local_out, lse, ep, s);
  return fwd_hd<128>(g, qkv, local_out, lse, ep, s);
}

cudaError_t launch_local_dq(const Geom& g, const void* qkv, const void* dl, const float* lse, const float* delta,
                            void* dqkv, cudaStream_t s) {
  if (((uintptr_t)qkv & 15) || ((uintptr_t)dl & 15) || ((uintptr_t)dqkv & 15)) return cudaErrorMisalignedAddress;
  if (g.hd == 64) return dq_hd<64>(g, qkv, dl, lse, delta, dqkv, s);
  return dq_hd<128>(g, qkv, dl, lse, delta, dqkv, s);
}

cudaError_t launch_local_dkv(const Geom& g, const void* qkv, const void* dl, const float* lse, const float* delta,
                             void* dqkv, cudaStream_t s) {
  if (((uintptr_t)qkv & 15) || ((uintptr_t)dl & 15) || ((uintptr_t)dqkv & 15)) return cudaErrorMisalignedAddress;
  if (g.hd == 64) return dkv_hd<64>(g, qkv, dl, lse, delta, dqkv, s);
  return dkv_hd<128>(g, qkv, dl, lse, delta, dqkv, s);
}

#if defined(LLATTN_TRACE)
extern "C" __attribute__((visibility("default"))) int llattn_trace_read(void* dst, size_t bytes) {
  return (int)cudaMemcpyFromSymbol(dst, g_trace, bytes < sizeof(g_trace) ? bytes : sizeof(g_trace));
}
#endif

unsigned read_fault_word(bool reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_fault_word, sizeof(v));
  if (reset) {
    unsigned z = 0;
    cudaMemcpyToSymbol(g_fault_word, &z, sizeof(z));
  }
  return v;
}

}  // namespace sm100
}  // namespace llattn
