// Local branch on the 5th-generation tensor cores (sm_100a): windowed causal
// attention with the reference's blockwise mask (models.py:232-305), bf16 in,
// fp32 accumulation in TMEM, head_dim 64 or 128.
//
// Forward, one CTA per (batch, head, 128-query tile), 6 warps:
//   warp 0     TMA producer: Q tile once, then K/V tiles of 128 keys into a
//              2-stage ring (tensor map over the qkv projection output
//              [B, T, 3, H, hd] read in place, 128-byte swizzle, OOB -> 0)
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer:
//              S_j = Q K_j^T (M128 N128, K = hd) into one of two TMEM S
//              buffers, then O += P_j V_j (M128 N=hd, K = 128 keys)
//   warps 2-5  softmax: thread r owns query row r = TMEM lane r. Reads S_j
//              from TMEM, applies the window mask and online softmax (exp2),
//              writes P_j (bf16, swizzled K-major) to shared memory, rescales
//              O in TMEM when the running max moves, and finally writes the
//              normalised row and its logsumexp.
// Key tiles start at lo(q0) (the first key any row of the tile sees), so a
// tile of 128 rows with window W touches ceil((127 + W) / 128) key tiles.
//
// Every wait is bounded (mbar_wait): on timeout the kernel records a fault
// bit in g_fault_word, tells the other warps to stop, frees its TMEM and
// returns; the host reads the word with llattn_fault_status().
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "sm100.cuh"
#include "sm100_ptx.cuh"

namespace llattn {
namespace sm100 {

// Nonzero once any tensor-core kernel gave up on a wait; every later wait
// (in any CTA) then returns at once, so a broken launch ends within about a
// second instead of timing out CTA by CTA.
__device__ unsigned int g_fault_word = 0;

namespace {

using namespace ptx;

constexpr int BM = 128;  // query rows per tile (= TMEM lanes)
constexpr int BN = 128;  // keys per tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum Fault : unsigned {
  kFaultProducer = 1u, kFaultMma = 2u, kFaultSoftmax = 4u, kFaultEpilogue = 8u,
};

__device__ __forceinline__ void raise_fault(unsigned bit, volatile int* abort) {
  atomicOr(&g_fault_word, bit);
  *abort = 1;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int HD>
struct FwdLayout {
  static constexpr int PANEL = BM * 128;       // 128 rows x 128 bytes (64 bf16)
  static constexpr int TILE = BM * HD * 2;      // one 128-row tile of hd columns
  static constexpr int Q = 0;
  static constexpr int K = Q + TILE;            // 2 stages
  static constexpr int V = K + 2 * TILE;        // 2 stages
  static constexpr int P = V + 2 * TILE;        // 128 x 128 bf16
  // the fused gate's lat tile (128 x 64 bf16) and W_rout slice (hd x 64 bf16)
  // live in the P region: the R MMA reads them before P_0 is written
  static constexpr int LAT = P;
  static constexpr int WR = P + BM * 128;
  static constexpr int XCH = P + BM * BN * 2;   // half-pair exchange, 2 x 2 x 128 x 2 floats
  static constexpr int BAR = XCH + 2 * 2 * BM * 2 * 4;
  static constexpr int BYTES = BAR + 256;
};

// Barrier slots in the BAR region.
enum { B_Q = 0, B_K = 1, B_V = 3, B_KVE = 5, B_S = 7, B_P = 9, B_O = 10, B_LW = 11, B_R = 12, B_X = 13,
       N_BARS = 17 };

template <int HD>
__global__ void __launch_bounds__(320, 1)
    local_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, Geom g, bf16* __restrict__ local_out,
                        float* __restrict__ lse_out, GateEpilogue ep) {
  using L = FwdLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + N_BARS);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * BM;
  const int qlast = min(q0 + BM - 1, g.T - 1);
  const int kbase = local_lo(g, q0);
  const int khi = qlast - 1;
  const int nk = khi >= kbase ? (khi - kbase + BN) / BN : 0;

  if (threadIdx.x == 0) {
    mbar_init(&bars[B_Q], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[B_K + s], 1);
      mbar_init(&bars[B_V + s], 1);
      mbar_init(&bars[B_KVE + s], 1);
      mbar_init(&bars[B_S + s], 1);
    }
    mbar_init(&bars[B_P], 2 * BM);
    mbar_init(&bars[B_O], 1);
    mbar_init(&bars[B_LW], 2 * BM);
    for (int q = 0; q < 4; ++q) mbar_init(&bars[B_X + q], 64);
    mbar_init(&bars[B_R], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS0 = tmem, tS1 = tmem + 128, tO = tmem + 256, tR = tmem + 256 + HD;
  const bool fuse = ep.lat != nullptr;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && nk > 0) {
      int issued = 0;
      prefetch_tmap(&tm_qkv);
      mbar_expect_tx(&bars[B_Q], L::TILE);
#pragma unroll
      for (int p = 0; p < HD / 64; ++p)
        tma_load_4d(&tm_qkv, &bars[B_Q], smem + L::Q + p * L::PANEL, p * 64, h, q0, b);
      for (int j = 0; j < nk; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bars[B_KVE + s], ((j >> 1) - 1) & 1, abort, &g_fault_word)) {
          raise_fault(kFaultProducer, abort);
          break;
        }
        const int k0 = kbase + j * BN;
        mbar_expect_tx(&bars[B_K + s], L::TILE);
#pragma unroll
        for (int p = 0; p < HD / 64; ++p)
          tma_load_4d(&tm_qkv, &bars[B_K + s], smem + L::K + s * L::TILE + p * L::PANEL, p * 64, g.H + h, k0, b);
        mbar_expect_tx(&bars[B_V + s], L::TILE);
#pragma unroll
        for (int p = 0; p < HD / 64; ++p)
          tma_load_4d(&tm_qkv, &bars[B_V + s], smem + L::V + s * L::TILE + p * L::PANEL, p * 64, 2 * g.H + h,
                      k0, b);
        issued = j + 1;
      }
      if (*abort) {
        // leave no bulk copy writing into shared memory after exit: wait
        // (bounded, ignoring the abort flags) for the last loads issued
        volatile int none = 0;
        volatile unsigned gnone = 0;
        mbar_wait(&bars[B_Q], 0, &none, &gnone, 100000000ull);
        for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
          mbar_wait(&bars[B_K + (j & 1)], (j >> 1) & 1, &none, &gnone, 100000000ull);
          mbar_wait(&bars[B_V + (j & 1)], (j >> 1) & 1, &none, &gnone, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && (nk > 0 || fuse)) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t idO = idesc_bf16_f32(BM, HD, false, true);
      const uint32_t q_addr = smem_u32(smem + L::Q);
      const uint32_t p_addr = smem_u32(smem + L::P);
      bool ok = true;
      if (fuse) {
        // remote tile R = lat_tile (128 x 64) . W_h^T (64 x hd), K-major both
        ok = mbar_wait(&bars[B_LW], 0, abort, &g_fault_word);
        if (ok) {
          tc_fence_after();
          constexpr uint32_t idR = idesc_bf16_f32(BM, HD, false, false);
          const uint32_t la = smem_u32(smem + L::LAT), wa = smem_u32(smem + L::WR);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tR, desc_sw128(la + kk * 32, 16, 1024), desc_sw128(wa + kk * 32, 16, 1024), idR, kk > 0);
          mma_commit(&bars[B_R]);
        }
      }
      if (ok && nk > 0) ok = mbar_wait(&bars[B_Q], 0, abort, &g_fault_word);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&bars[B_K + s], (j >> 1) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::K + s * L::TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk / 4) * L::PANEL + (kk % 4) * 32;
          mma_bf16(s ? tS1 : tS0, desc_sw128(q_addr + off, 16, 1024), desc_sw128(k_addr + off, 16, 1024), idS,
                   kk > 0);
        }
        mma_commit(&bars[B_S + s]);
        return true;
      };
      if (ok && nk > 0) ok = issue_s(0);
      for (int j = 0; ok && j < nk; ++j) {
        if (j + 1 < nk && !(ok = issue_s(j + 1))) break;
        if (!(ok = mbar_wait(&bars[B_P], j & 1, abort, &g_fault_word))) break;
        if (!(ok = mbar_wait(&bars[B_V + (j & 1)], (j >> 1) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + L::V + (j & 1) * L::TILE);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t a = desc_sw128(p_addr + (kk / 4) * L::PANEL + (kk % 4) * 32, 16, 1024);
          const uint64_t bdesc = desc_sw128(v_addr + kk * 16 * 128, L::PANEL, 1024);
          mma_bf16(tO, a, bdesc, idO, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars[B_KVE + (j & 1)]);
        mma_commit(&bars[B_O]);
      }
      if (!ok) raise_fault(kFaultMma, abort);
    }
  } else {
    // ---------------- softmax / epilogue (warps 2..9) ----------------
    // Row r = TMEM lane r is shared by warps w and w+4 (same lane quarter):
    // half 0 owns key columns [0,64) and O columns [0,hd/2), half 1 the rest.
    // The pair exchanges row maxima / sums through shared memory guarded by
    // a per-quarter mbarrier (64 arrivals per use, bounded waits).
    const int half = (warp - 2) >> 2, quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const int t = q0 + row;
    const bool valid = t < g.T;
    const int lo = valid ? local_lo(g, t) : 0x7fffffff;
    const float sc = g.scale * kLog2e;
    float m = -INFINITY, l = 0.f;  // l: this half's partial row sum
    uint8_t* prow = smem + L::P + row * 128;
    float* xch = reinterpret_cast<float*>(smem + L::XCH);  // [2 bufs][2 halves][128 rows][2]
    int xuse = 0;
    // publish (a, b) for this row, receive the partner half's pair
    auto exchange = [&](float a, float bv, float& pa, float& pb) -> bool {
      float* mine = xch + (((xuse & 1) * 2 + half) * BM + row) * 2;
      float* other = xch + (((xuse & 1) * 2 + (half ^ 1)) * BM + row) * 2;
      mine[0] = a;
      mine[1] = bv;
      mbar_arrive(&bars[B_X + quarter]);
      const bool okx = __all_sync(0xffffffffu, mbar_wait(&bars[B_X + quarter], xuse & 1, abort, &g_fault_word));
      pa = other[0];
      pb = other[1];
      ++xuse;
      return okx;
    };
    bool ok = true;
    if (fuse) {
      // row `row` of the lat tile (half 0) and of W_rout's head slice (half 1,
      // rows < hd): 128-byte rows, 16-byte chunk c at slot c ^ (row % 8)
      if (half == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const bf16*>(ep.lat) +
                                                          ((int64_t)b * g.Tq + (valid ? t / g.qbs : 0)) * 64);
        uint8_t* dl_ = smem + L::LAT + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dl_ + ((c ^ (row & 7)) * 16)) = src[c];
      } else if (row < HD) {
        const uint4* wsrc = reinterpret_cast<const uint4*>(static_cast<const bf16*>(ep.w_rout) +
                                                           ((int64_t)h * HD + row) * 64);
        uint8_t* wd = smem + L::WR + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(wd + ((c ^ (row & 7)) * 16)) = wsrc[c];
      }
      fence_async_smem();
      mbar_arrive(&bars[B_LW]);
      // P_0 overwrites this region: wait until the R MMA has read it
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_R], 0, abort, &g_fault_word));
    }
    for (int j = 0; ok && j < nk; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_S + s], (j >> 1) & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tsrc = (s ? tS1 : tS0) + lane_off + half * 64;
      const int c_lo = lo - (kbase + j * BN) - half * 64;  // visible columns of this half: [c_lo, c_hi)
      const int c_hi = t - (kbase + j * BN) - half * 64;
      // pass 1: masked row max over this half's 64 columns, then both halves
      float mx = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        tmem_ld32(tsrc + cc * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = cc * 32 + i;
          if (c >= c_lo && c < c_hi) mx = fmaxf(mx, __uint_as_float(r[i]));
        }
      }
      float pmx, unused;
      if (!(ok = exchange(mx, 0.f, pmx, unused))) break;
      mx = fmaxf(mx, pmx);
      const float m_new = fmaxf(m, mx * sc);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);
      // P buffer and O are free once PV_{j-1} has completed
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_O], (j - 1) & 1, abort, &g_fault_word));
        if (!ok) break;
      }
      tc_fence_after();
      // pass 2: p = exp2(s*sc - m), bf16, swizzled store into panel `half`
      float psum = 0.f;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        tmem_ld32(tsrc + cc * 32, r);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = cc * 32 + 2 * i;
          const float p0 = (c >= c_lo && c < c_hi) ? exp2f(__uint_as_float(r[2 * i]) * sc - m_use) : 0.f;
          const float p1 =
              (c + 1 >= c_lo && c + 1 < c_hi) ? exp2f(__uint_as_float(r[2 * i + 1]) * sc - m_use) : 0.f;
          psum += p0 + p1;
          pk[i] = pack_bf16(p0, p1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = cc * 4 + q;
          const int slot = (chunk & 7) ^ (row & 7);
          *reinterpret_cast<uint4*>(prow + half * L::PANEL + slot * 16) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      fence_async_smem();
      l = l * alpha + psum;
      m = m_new;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int cc = 0; cc < HD / 64; ++cc) {
          uint32_t r[32];
          const uint32_t ta = tO + lane_off + half * (HD / 2) + cc * 32;
          tmem_ld32(ta, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(ta, r);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(&bars[B_P]);
    }
    if (!ok) raise_fault(kFaultSoftmax, abort);
    // epilogue. The TMEM loads are warp-collective (.sync.aligned): every
    // lane executes them, rows past T only skip the stores.
    if (ok && nk > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_O], (nk - 1) & 1, abort, &g_fault_word));
    float pl = 0.f, unused2;
    if (ok) ok = exchange(l, 0.f, pl, unused2);
    if (!ok) {
      raise_fault(kFaultEpilogue, abort);
    } else {
      tc_fence_after();
      l += pl;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int c0 = half * (HD / 2);  // this half's O columns
      bf16* dst = local_out + ((int64_t)b * g.T + (valid ? t : 0)) * g.d + (int64_t)h * HD + c0;
      if (fuse) {
        // pass A: gate logits from the bf16-rounded local row (the value
        // stored for the backward) and the remote row, halves combined
        const float4* bh4 = reinterpret_cast<const float4*>(ep.b_rout + (int64_t)h * HD + c0);
        const float4* gl4 = reinterpret_cast<const float4*>(ep.g_local + c0);
        const float4* gr4 = reinterpret_cast<const float4*>(ep.g_remote + c0);
        float sl = 0.f, sr = 0.f;
#pragma unroll
        for (int cc = 0; cc < HD / 64; ++cc) {
          uint32_t ro[32], rr[32];
          if (nk > 0) tmem_ld32(tO + lane_off + c0 + cc * 32, ro);
          tmem_ld32(tR + lane_off + c0 + cc * 32, rr);
          tmem_ld_wait();
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const float4 bb = __ldg(bh4 + cc * 8 + i4), ga = __ldg(gl4 + cc * 8 + i4), gb = __ldg(gr4 + cc * 8 + i4);
            const float bv[4] = {bb.x, bb.y, bb.z, bb.w}, gav[4] = {ga.x, ga.y, ga.z, ga.w};
            const float gbv[4] = {gb.x, gb.y, gb.z, gb.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int i = 4 * i4 + k;
              const float lv = nk > 0 ? __bfloat162float(__float2bfloat16_rn(__uint_as_float(ro[i]) * inv)) : 0.f;
              sl = fmaf(lv, gav[k], sl);
              sr = fmaf(__uint_as_float(rr[i]) + bv[k], gbv[k], sr);
            }
          }
        }
        float psl, psr;
        if (!exchange(sl, sr, psl, psr)) {
          raise_fault(kFaultEpilogue, abort);
        } else {
          const float x = sl + psl + g.gate_bias - (sr + psr);
          const float wl = 1.f / (1.f + expf(-x));
          const float wr = 1.f / (1.f + expf(x));
          bf16* mdst =
              static_cast<bf16*>(ep.mixed) + ((int64_t)b * g.T + (valid ? t : 0)) * g.d + (int64_t)h * HD + c0;
          // pass B: local_out and mixed
#pragma unroll
          for (int cc = 0; cc < HD / 64; ++cc) {
            uint32_t ro[32], rr[32];
            if (nk > 0) tmem_ld32(tO + lane_off + c0 + cc * 32, ro);
            tmem_ld32(tR + lane_off + c0 + cc * 32, rr);
            tmem_ld_wait();
            uint32_t plk[16], pm[16];
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
              const float4 bb = __ldg(bh4 + cc * 8 + i4);
              const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
              float lv[4], mv[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int i = 4 * i4 + k;
                lv[k] = nk > 0 ? __bfloat162float(__float2bfloat16_rn(__uint_as_float(ro[i]) * inv)) : 0.f;
                mv[k] = wl * lv[k] + wr * (__uint_as_float(rr[i]) + bv[k]);
              }
              plk[2 * i4] = pack_bf16(lv[0], lv[1]);
              plk[2 * i4 + 1] = pack_bf16(lv[2], lv[3]);
              pm[2 * i4] = pack_bf16(mv[0], mv[1]);
              pm[2 * i4 + 1] = pack_bf16(mv[2], mv[3]);
            }
            if (valid) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                *reinterpret_cast<uint4*>(dst + cc * 32 + q * 8) =
                    make_uint4(plk[4 * q], plk[4 * q + 1], plk[4 * q + 2], plk[4 * q + 3]);
                *reinterpret_cast<uint4*>(mdst + cc * 32 + q * 8) =
                    make_uint4(pm[4 * q], pm[4 * q + 1], pm[4 * q + 2], pm[4 * q + 3]);
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int cc = 0; cc < HD / 64; ++cc) {
          uint32_t r[32];
          if (nk > 0) {
            tmem_ld32(tO + lane_off + c0 + cc * 32, r);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack_bf16(__uint_as_float(r[2 * i]) * inv, __uint_as_float(r[2 * i + 1]) * inv);
          if (valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(dst + cc * 32 + q * 8) =
                  make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
        }
      }
      if (valid && half == 0)
        lse_out[((int64_t)b * g.H + h) * g.T + t] = l > 0.f ? (m + log2f(l)) * kLn2 : INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();  // lane 0 issued the MMAs alone; dealloc is warp-collective
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

#include "local_sm100_bwd.cuh"
#include "gate_sm100.cuh"

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

// [B, T, S, H, hd] bf16 viewed as 4-D (hd, S*H, T, B); box (64, 1, rows, 1).
bool make_rows_map(CUtensorMap* map, const void* base, int B, int T, int slots_x_heads, int hd, int rows = 128) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)hd, (cuuint64_t)slots_x_heads, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)hd * 2, (cuuint64_t)slots_x_heads * hd * 2,
                           (cuuint64_t)T * slots_x_heads * hd * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool force_simt() {
  const char* e = std::getenv("LLATTN_FORCE_SIMT");
  return e && e[0] == '1';
}

template <int HD>
cudaError_t fwd_hd(const Geom& g, const void* qkv, void* local_out, float* lse, const GateEpilogue& ep,
                   cudaStream_t s) {
  CUtensorMap tm;
  if (!make_rows_map(&tm, qkv, g.B, g.T, 3 * g.H, HD)) return cudaErrorInvalidValue;
  // at least 116 KB so a second CTA never shares the SM (and its TMEM)
  const int smem = std::max(FwdLayout<HD>::BYTES + 1024, 116 * 1024);
  cudaError_t e = cudaFuncSetAttribute(local_fwd_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, BM), g.H, g.B);
  local_fwd_tc_kernel<HD><<<grid, 320, smem, s>>>(tm, g, static_cast<bf16*>(local_out), lse, ep);
  return cudaGetLastError();
}

template <int HD>
cudaError_t dq_hd(const Geom& g, const void* qkv, const void* dl, const float* lse, const float* delta, void* dqkv,
                  cudaStream_t s) {
  CUtensorMap q128, q64, do128;
  if (!make_rows_map(&q128, qkv, g.B, g.T, 3 * g.H, HD, 128) || !make_rows_map(&q64, qkv, g.B, g.T, 3 * g.H, HD, 64) ||
      !make_rows_map(&do128, dl, g.B, g.T, g.H, HD, 128))
    return cudaErrorInvalidValue;
  const int smem = std::max(DqLayout<HD>::BYTES + 1024, 116 * 1024);
  cudaError_t e = cudaFuncSetAttribute(local_dq_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, BM), g.H, g.B);
  local_dq_tc_kernel<HD><<<grid, 320, smem, s>>>(q128, q64, do128, g, lse, delta, static_cast<bf16*>(dqkv));
  return cudaGetLastError();
}

template <int HD>
cudaError_t dkv_hd(const Geom& g, const void* qkv, const void* dl, const float* lse, const float* delta, void* dqkv,
                   cudaStream_t s) {
  CUtensorMap q128, q64, do64;
  if (!make_rows_map(&q128, qkv, g.B, g.T, 3 * g.H, HD, 128) || !make_rows_map(&q64, qkv, g.B, g.T, 3 * g.H, HD, 64) ||
      !make_rows_map(&do64, dl, g.B, g.T, g.H, HD, 64))
    return cudaErrorInvalidValue;
  const int smem = std::max(DkvLayout<HD>::BYTES + 1024, 116 * 1024);
  cudaError_t e = cudaFuncSetAttribute(local_dkv_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, BM), g.H, g.B);
  local_dkv_tc_kernel<HD><<<grid, 320, smem, s>>>(q128, q64, do64, g, lse, delta, static_cast<bf16*>(dqkv));
  return cudaGetLastError();
}

template <int HD>
cudaError_t gate_bwd_hd(const Geom& g, const GateBwd& a, cudaStream_t s) {
  CUtensorMap tlo, tdm;
  if (!make_2d_map(&tlo, a.local_out, (int64_t)g.B * g.T, g.d, 128) ||
      !make_2d_map(&tdm, a.dmixed, (int64_t)g.B * g.T, g.d, 128))
    return cudaErrorInvalidValue;
  const int smem = std::max(GbLayout<HD>::BYTES + 1024, 116 * 1024);
  cudaError_t e = cudaFuncSetAttribute(gate_bwd_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.T, BM), g.B);
  gate_bwd_tc_kernel<HD><<<grid, 320, smem, s>>>(
      tlo, tdm, g, static_cast<const bf16*>(a.local_out), static_cast<const bf16*>(a.lat), static_cast<const bf16*>(a.w_rout),
      a.b_rout, a.g_local, a.g_remote, static_cast<const bf16*>(a.dmixed), static_cast<bf16*>(a.dl), a.delta,
      static_cast<bf16*>(a.dr), a.dlat_tok, a.dg_part);
  return cudaGetLastError();
}

}  // namespace

int gate_bwd_ctas(const Geom& g) { return g.B * cdiv(g.T, BM); }

cudaError_t launch_gate_bwd(const Geom& g, const GateBwd& a, cudaStream_t s) {
  if (g.hd == 64) return gate_bwd_hd<64>(g, a, s);
  return gate_bwd_hd<128>(g, a, s);
}

cudaError_t launch_rout_dw(const Geom& g, const void* dr, const void* lat, float* dw_part, float* db_part,
                           int n_split, cudaStream_t s) {
  CUtensorMap tm;
  if (!make_2d_map(&tm, dr, (int64_t)g.B * g.T, g.d)) return cudaErrorInvalidValue;
  const int smem = std::max(DwLayout::BYTES + 1024, 116 * 1024);
  cudaError_t e = cudaFuncSetAttribute(rout_dw_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.d, 128), n_split);
  rout_dw_tc_kernel<<<grid, 192, smem, s>>>(tm, g, static_cast<const bf16*>(lat), dw_part, db_part, n_split);
  return cudaGetLastError();
}

cudaError_t launch_dlat_rowsum(const Geom& g, const float* dlat_tok, float* dlat, cudaStream_t s) {
  const int64_t n = (int64_t)g.B * g.Tq * 64;
  dlat_rowsum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, dlat_tok, dlat);
  return cudaGetLastError();
}

bool fwd_supported(const Geom& g, int elt_bytes) {
  return !force_simt() && elt_bytes == 2 && (g.hd == 64 || g.hd == 128) && get_encode() != nullptr;
}

bool bwd_supported(const Geom& g, int elt_bytes) { return fwd_supported(g, elt_bytes); }

bool gate_fusable(const Geom& g) { return g.Ld == 64; }

cudaError_t launch_local_fwd(const Geom& g, const void* qkv, void* local_out, float* lse, const GateEpilogue& ep,
                             cudaStream_t s) {
  if (((uintptr_t)qkv & 15) || ((uintptr_t)local_out & 15)) return cudaErrorMisalignedAddress;
  if (ep.lat && (g.Ld != 64 || ((uintptr_t)ep.lat & 15) || ((uintptr_t)ep.w_rout & 15) ||
                 ((uintptr_t)ep.mixed & 15)))
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
