// Latent-branch kernels on the tensor cores (included by local_sm100.cu),
// bf16 activations, latent head dims up to 64: for at most 64 chunks a
// backward and a forward that hold one key tile; past 64 chunks (up to 512)
// a two-pass forward and a rows / keys backward pair, further down.
//
// Backward for at most 64 chunks (one key tile), bf16 activations and
// latent head dims up to 64: LDH = 32, or 64 for 32 < ldh <= 64 (ldh a
// multiple of 8; the columns past ldh are zero in every operand). Math as
// the SIMT kernel of latent.cu: with P = softmax(lat_scale rq.gk) over chunks
// j < qid(r) (models.py:361-375), dP = dlat.gv, delta = sum_j P dP,
// dS = P (dP - delta):
//   drq = lat_scale dS gk,  dgk = lat_scale dS^T rq,  dgv = P^T dlat.
//
// CTA = (row split, latent head, b); it walks the 128-row tiles
// rb = split + k * n_split of its (b, head). Warps 0-3: thread = row = TMEM
// lane (operand rows in, softmax, drq out); warp 4: TMEM allocation and the
// single MMA-issuing thread. Per tile:
//   1. S = rq gk^T and dP = dlat gv^T as kind::tf32 MMAs (fp32 operands: dlat
//      keeps 11 mantissa bits, since dP - delta cancels when the pooled values
//      are close; rq and gk are bf16 values, exact in tf32)
//   2. the threads form P, delta, dS in fp32; dS goes to TMEM as bf16 (A of
//      the drq MMA) and both dS and P to shared memory as bf16
//   3. drq = dS gk with A from TMEM, and D2 += [rq | dlat]^T [dS | P] over
//      the tile's rows (M = 128, N = 128, both operands MN-major): rows
//      e < LDH x columns j < 64 are dgk^T / lat_scale, rows LDH + e x columns
//      64 + j are dgv^T (LDH = 32: rows 64-127 come from unrelated bytes and
//      are never read). D2 stays in TMEM across the CTA's tiles and is
//      written once as the CTA's partial.
// Everything within a tile is sequential; two CTAs per SM overlap each other.

template <int LDH>
struct LatTcLayout {
  static constexpr int FP = LDH / 32;           // 128-byte panels of an fp32 row
  static constexpr int AS = 0;                  // rq fp32 [128 rows][LDH] (K-major, tf32), FP panels of 16 KB
  static constexpr int AD = AS + FP * 16384;    // dlat fp32 [128][LDH]
  // [128 rows][rq bf16 | dlat bf16] (MN-major A of D2): LDH 32 one 128-byte
  // row, LDH 64 a rq panel and a dlat panel of 16 KB
  static constexpr int X = AD + FP * 16384;
  static constexpr int BP = X + (LDH == 64 ? 32768 : 16384);  // dS bf16 [128 rows][64 keys], then P at +16 KB
  static constexpr int GK = BP + 32768;         // gk fp32 [64 keys][LDH], FP panels of 8 KB
  static constexpr int GV = GK + FP * 8192;     // gv fp32 [64][LDH]
  static constexpr int GKB = GV + FP * 8192;    // gk bf16 [64 keys][LDH] in 128-byte rows (MN-major B of drq)
  static constexpr int BAR = GKB + 8192;
  static constexpr int BYTES = BAR + 128;
  static_assert(LDH == 64 || BYTES + 1024 <= 113 * 1024, "two CTAs per SM");
  static_assert(BYTES + 1024 <= 227 * 1024, "shared memory");
};

enum { LT_A = 0, LT_S = 1, LT_P = 2, LT_T = 3, LT_NB = 4 };

__device__ __forceinline__ uint4* lat_chunk(uint8_t* tile, int row, int c) {  // 16-byte chunk c of a 128-byte row
  return reinterpret_cast<uint4*>(tile + row * 128 + ((c ^ (row & 7)) * 16));
}
// chunk c (16 bytes) of a row that spans several 128-byte panels of `rows` rows
__device__ __forceinline__ uint4* lat_pchunk(uint8_t* tile, int rows, int row, int c) {
  return lat_chunk(tile + (c >> 3) * rows * 128, row, c & 7);
}

template <int LDH>
__global__ void __launch_bounds__(160, LDH == 32 ? 2 : 1)
    latent_bwd_tc_kernel(Geom g, const bf16* __restrict__ rq, const bf16* __restrict__ gkv,
                         const float* __restrict__ lat_lse, const float* __restrict__ dlat, bf16* __restrict__ drq,
                         float* __restrict__ part, int n_split) {
  using L = LatTcLayout<LDH>;
  constexpr int NQ = LDH / 8, ND = LDH / 4;  // 16-byte chunks of a bf16 / fp32 row
  extern __shared__ __align__(1024) uint8_t smem_lat_tc[];
  uint8_t* smem = smem_lat_tc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + LT_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int split = blockIdx.x, lh = blockIdx.y, b = blockIdx.z;
  const int n_rb = cdiv(g.Tq, BM);
  const int n_tiles = split < n_rb ? (n_rb - 1 - split) / n_split + 1 : 0;
  const int ldh = g.ldh;  // <= LDH, a multiple of 8: chunks past it are zero

  if (tid == 0) {
    mbar_init(&bars[LT_A], BM);
    mbar_init(&bars[LT_S], 1);
    mbar_init(&bars[LT_P], BM);
    mbar_init(&bars[LT_T], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    __syncwarp();
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  // chunk keys / values of (b, lh): thread = (key, half of the LDH dims)
  if (tid < BM) {
    const int key = tid >> 1, c0 = (tid & 1) * (NQ / 2);  // first bf16 chunk of this half
    const bf16* kp = gkv + ((int64_t)(b * g.Nc + key) * 2 * g.Lh + lh) * ldh;
    const bf16* vp = gkv + ((int64_t)(b * g.Nc + key) * 2 * g.Lh + g.Lh + lh) * ldh;
#pragma unroll
    for (int q = 0; q < NQ / 2; ++q) {
      const int c = c0 + q;  // bf16 chunk: elements 8c .. 8c+7
      const bool on = key < g.Nc && 8 * c < ldh;
      const uint4 k2 = on ? reinterpret_cast<const uint4*>(kp)[c] : make_uint4(0, 0, 0, 0);
      const uint4 v2 = on ? reinterpret_cast<const uint4*>(vp)[c] : make_uint4(0, 0, 0, 0);
      float kf[8], vf[8];
      unpack8(k2, kf);
      unpack8(v2, vf);
      *lat_pchunk(smem + L::GK, 64, key, 2 * c) = make_uint4(__float_as_uint(kf[0]), __float_as_uint(kf[1]),
                                                             __float_as_uint(kf[2]), __float_as_uint(kf[3]));
      *lat_pchunk(smem + L::GK, 64, key, 2 * c + 1) = make_uint4(__float_as_uint(kf[4]), __float_as_uint(kf[5]),
                                                                 __float_as_uint(kf[6]), __float_as_uint(kf[7]));
      *lat_pchunk(smem + L::GV, 64, key, 2 * c) = make_uint4(__float_as_uint(vf[0]), __float_as_uint(vf[1]),
                                                             __float_as_uint(vf[2]), __float_as_uint(vf[3]));
      *lat_pchunk(smem + L::GV, 64, key, 2 * c + 1) = make_uint4(__float_as_uint(vf[4]), __float_as_uint(vf[5]),
                                                                 __float_as_uint(vf[6]), __float_as_uint(vf[7]));
      *lat_chunk(smem + L::GKB, key, c) = k2;
    }
    if (LDH == 32)  // the drq MMA reads 64 columns of gk bf16: the upper half is zero
#pragma unroll
      for (int q = 0; q < 2; ++q) *lat_chunk(smem + L::GKB, key, 4 + (tid & 1) * 2 + q) = make_uint4(0, 0, 0, 0);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: S [0,64) (then drq), dP [64,128) with dS bf16 over [64,96), D2 [128,256)
  const uint32_t tS = tmem, tP = tmem + 64, tD2 = tmem + 128;

  if (warp == 4) {
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t id1 = idesc_tf32_f32(BM, 64);
      constexpr uint32_t idQ = idesc_bf16_f32(BM, 64, false, true);   // dS gk
      constexpr uint32_t id2 = idesc_bf16_f32(BM, 128, true, true);   // [rq | dlat]^T [dS | P]
      const uint64_t das = desc_sw128(smem_u32(smem + L::AS), 16, 1024);
      const uint64_t dad = desc_sw128(smem_u32(smem + L::AD), 16, 1024);
      const uint64_t dgk = desc_sw128(smem_u32(smem + L::GK), 16, 1024);
      const uint64_t dgv = desc_sw128(smem_u32(smem + L::GV), 16, 1024);
      const uint64_t dkb = desc_sw128(smem_u32(smem + L::GKB), 8192, 1024);
      // LDH 32: M = 128 reads a second 64-row panel of A 16 KB on (the dS
      // tile): the D2 rows it produces (64-127) are never read
      const uint64_t dx = desc_sw128(smem_u32(smem + L::X), 16384, 1024);
      const uint64_t dbp = desc_sw128(smem_u32(smem + L::BP), 16384, 1024);
      bool ok = true;
      for (int n = 0; ok && n < n_tiles; ++n) {
        if (!(ok = mbar_wait(&bars[LT_A], n & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        // K steps of 8 fp32 (32 bytes); panels of 32 fp32 at 16 KB (A) / 8 KB (B)
#pragma unroll
        for (int kk = 0; kk < LDH / 8; ++kk) {
          const uint32_t ao = (kk / 4) * 16384 + (kk % 4) * 32, bo = (kk / 4) * 8192 + (kk % 4) * 32;
          mma_tf32(tS, desc_add(das, ao), desc_add(dgk, bo), id1, kk > 0);
          mma_tf32(tP, desc_add(dad, ao), desc_add(dgv, bo), id1, kk > 0);
        }
        mma_commit(&bars[LT_S]);
        if (!(ok = mbar_wait(&bars[LT_P], n & 1, abort, &g_fault_word))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma_bf16_ts(tS, tP + kk * 8, desc_add(dkb, kk * 2048), idQ, kk > 0);
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          mma_bf16(tD2, desc_add(dx, kk * 2048), desc_add(dbp, kk * 2048), id2, (n > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars[LT_T]);
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const float sc2 = g.lat_scale * kLog2e;
    uint4 pre_q[NQ], pre_d[ND];  // next tile's rq (bf16) / dlat (fp32) row
    float pre_lse = INFINITY;
    auto fetch = [&](int n) {
      const int r = (split + n * n_split) * BM + tid;
      const bool on = n < n_tiles && r < g.Tq;
      const uint4* qp = reinterpret_cast<const uint4*>(rq + ((int64_t)(b * g.Tq + (on ? r : 0)) * g.Lh + lh) * ldh);
      const uint4* dp = reinterpret_cast<const uint4*>(dlat + (int64_t)(b * g.Tq + (on ? r : 0)) * g.Ld + lh * ldh);
#pragma unroll
      for (int i = 0; i < NQ; ++i) pre_q[i] = (on && 8 * i < ldh) ? __ldg(qp + i) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < ND; ++i) pre_d[i] = (on && 4 * i < ldh) ? __ldg(dp + i) : make_uint4(0, 0, 0, 0);
      pre_lse = on ? __ldg(lat_lse + (int64_t)(b * g.Lh + lh) * g.Tq + r) * kLog2e : INFINITY;
    };
    fetch(0);
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int r = (split + n * n_split) * BM + tid;
      const bool valid = r < g.Tq;
      const int qid = valid ? row_qid(g, r) : 0;
      const float lse2 = pre_lse;
      // operands of this tile (the previous tile's MMAs finished reading them)
      if (n > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[LT_T], (n - 1) & 1, abort, &g_fault_word));
        if (!ok) break;
      }
#pragma unroll
      for (int c = 0; c < ND; ++c) *lat_pchunk(smem + L::AD, BM, tid, c) = pre_d[c];
#pragma unroll
      for (int i = 0; i < NQ; ++i) {
        float f[8];
        unpack8(pre_q[i], f);
        *lat_pchunk(smem + L::AS, BM, tid, 2 * i) = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                                                               __float_as_uint(f[2]), __float_as_uint(f[3]));
        *lat_pchunk(smem + L::AS, BM, tid, 2 * i + 1) = make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]),
                                                                   __float_as_uint(f[6]), __float_as_uint(f[7]));
        *lat_pchunk(smem + L::X, BM, tid, i) = pre_q[i];
        const float4 d0 = *reinterpret_cast<const float4*>(&pre_d[2 * i]);
        const float4 d1 = *reinterpret_cast<const float4*>(&pre_d[2 * i + 1]);
        *lat_pchunk(smem + L::X, BM, tid, NQ + i) = make_uint4(pack_bf16(d0.x, d0.y), pack_bf16(d0.z, d0.w),
                                                               pack_bf16(d1.x, d1.y), pack_bf16(d1.z, d1.w));
      }
      fence_async_smem();
      mbar_arrive(&bars[LT_A]);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[LT_S], n & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      // P and dP of this row: keys in two halves of 32
      float p[64], dp[64];
      {
        uint32_t rs[32], rp[32];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          tmem_ld32(tS + lane_off + hh * 32, rs);
          tmem_ld32(tP + lane_off + hh * 32, rp);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int j = hh * 32 + i;
            p[j] = j < qid ? fast_exp2(fmaf(__uint_as_float(rs[i]), sc2, -lse2)) : 0.f;
            dp[j] = __uint_as_float(rp[i]);
          }
        }
      }
      float delta = 0.f;
#pragma unroll
      for (int j = 0; j < 64; ++j) delta = fmaf(p[j], dp[j], delta);
      uint32_t pk[32], pp[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        pk[i] = pack_bf16(p[2 * i] * (dp[2 * i] - delta), p[2 * i + 1] * (dp[2 * i + 1] - delta));
        pp[i] = pack_bf16(p[2 * i], p[2 * i + 1]);
      }
      {
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          lo[i] = pk[i];
          hi[i] = pk[16 + i];
        }
        tmem_st16(tP + lane_off, lo);
        tmem_st16(tP + lane_off + 16, hi);
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        *lat_chunk(smem + L::BP, tid, c) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *lat_chunk(smem + L::BP + 16384, tid, c) = make_uint4(pp[4 * c], pp[4 * c + 1], pp[4 * c + 2], pp[4 * c + 3]);
      }
      tmem_st_wait();
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[LT_P]);
      fetch(n + 1);  // next tile's rows load during this tile's MMAs
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[LT_T], n & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      uint32_t rq32[32];
#pragma unroll
      for (int hh = 0; hh < LDH / 32; ++hh) {
        tmem_ld32(tS + lane_off + hh * 32, rq32);
        tmem_ld_wait();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(drq + ((int64_t)(b * g.Tq + r) * g.Lh + lh) * ldh + hh * 32);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (hh * 32 + 8 * c < ldh)
              dst[c] = make_uint4(pack_bf16(__uint_as_float(rq32[8 * c]) * g.lat_scale,
                                            __uint_as_float(rq32[8 * c + 1]) * g.lat_scale),
                                  pack_bf16(__uint_as_float(rq32[8 * c + 2]) * g.lat_scale,
                                            __uint_as_float(rq32[8 * c + 3]) * g.lat_scale),
                                  pack_bf16(__uint_as_float(rq32[8 * c + 4]) * g.lat_scale,
                                            __uint_as_float(rq32[8 * c + 5]) * g.lat_scale),
                                  pack_bf16(__uint_as_float(rq32[8 * c + 6]) * g.lat_scale,
                                            __uint_as_float(rq32[8 * c + 7]) * g.lat_scale));
        }
      }
    }
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
    // this CTA's dgk / dgv partial: D2 row m = 32 warp + lane is dgk^T row e
    // for m < LDH and dgv^T row m - LDH after it (LDH 32: rows >= 64 unused);
    // partial layout [split][b][key][2][Ld]
    const int m = 32 * warp + lane, which = m / LDH, e = m % LDH;
    if (which < 2) {
      float* my_part = part + ((int64_t)split * g.B + b) * g.Nc * 2 * g.Ld + lh * ldh + e;
      const float mul = which == 0 ? g.lat_scale : 1.f;
      const bool have = ok && n_tiles > 0 && !*abort;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t v[32];
        if (have) {
          tmem_ld32(tD2 + lane_off + which * 64 + hh * 32, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
        if (e < ldh) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = hh * 32 + i;
            if (key < g.Nc) my_part[(int64_t)(2 * key + which) * g.Ld] = __uint_as_float(v[i]) * mul;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// Forward of the latent branch on the tensor cores (same conditions): per
// 128-row tile, S = rq gk^T (bf16 operands, fp32 accumulation), the
// threads mask chunks j >= qid(r), take the row max and P = 2^(S sc - max) in
// fp32 (the normaliser l sums the fp32 P), and write P as bf16 over the S
// columns; lat = (P gv) / l, lat_lse = max + ln l (INFINITY and lat = 0 for
// rows that see no chunk, models.py:366-373). gk and gv sit in 128-byte rows
// (columns past ldh zero): K-major B of the score MMA and MN-major B of P gv.
struct LatFwdTcLayout {
  static constexpr int AQ = 0;              // rq bf16 [128 rows][<= 64] in 128-byte rows
  static constexpr int GK = AQ + 16384;     // gk bf16 [64 keys][<= 64]
  static constexpr int GV = GK + 8192;      // gv bf16 [64 keys][<= 64]
  static constexpr int BAR = GV + 8192;
  static constexpr int BYTES = BAR + 128;
};

template <int LDH>
__global__ void __launch_bounds__(160)
    latent_fwd_tc_kernel(Geom g, const bf16* __restrict__ rq, const bf16* __restrict__ gkv, bf16* __restrict__ lat,
                         float* __restrict__ lat_lse, int n_split) {
  using L = LatFwdTcLayout;
  constexpr int NQ = LDH / 8;
  extern __shared__ __align__(1024) uint8_t smem_latf_tc[];
  uint8_t* smem = smem_latf_tc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + LT_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int split = blockIdx.x, lh = blockIdx.y, b = blockIdx.z;
  const int n_rb = cdiv(g.Tq, BM);
  const int n_tiles = split < n_rb ? (n_rb - 1 - split) / n_split + 1 : 0;
  const int ldh = g.ldh;

  if (tid == 0) {
    mbar_init(&bars[LT_A], BM);
    mbar_init(&bars[LT_S], 1);
    mbar_init(&bars[LT_P], BM);
    mbar_init(&bars[LT_T], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    __syncwarp();
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  if (tid < BM) {  // chunk keys / values of (b, lh): thread = (key, half of the row's 8 chunks)
    const int key = tid >> 1, c0 = (tid & 1) * 4;
    const bf16* kp = gkv + ((int64_t)(b * g.Nc + key) * 2 * g.Lh + lh) * ldh;
    const bf16* vp = gkv + ((int64_t)(b * g.Nc + key) * 2 * g.Lh + g.Lh + lh) * ldh;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = c0 + q;
      const bool on = key < g.Nc && 8 * c < ldh;
      *lat_chunk(smem + L::GK, key, c) = on ? reinterpret_cast<const uint4*>(kp)[c] : make_uint4(0, 0, 0, 0);
      *lat_chunk(smem + L::GV, key, c) = on ? reinterpret_cast<const uint4*>(vp)[c] : make_uint4(0, 0, 0, 0);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 64;  // S [0,64) with P bf16 over [0,32); P gv at [64,128)

  if (warp == 4) {
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, 64, false, false);  // rq gk^T
      constexpr uint32_t idO = idesc_bf16_f32(BM, 64, false, true);   // P gv
      const uint64_t daq = desc_sw128(smem_u32(smem + L::AQ), 16, 1024);
      const uint64_t dk = desc_sw128(smem_u32(smem + L::GK), 16, 1024);
      const uint64_t dv = desc_sw128(smem_u32(smem + L::GV), 8192, 1024);
      bool ok = true;
      for (int n = 0; ok && n < n_tiles; ++n) {
        if (!(ok = mbar_wait(&bars[LT_A], n & 1, abort, &g_fault_word))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < LDH / 16; ++kk)
          mma_bf16(tS, desc_add(daq, kk * 32), desc_add(dk, kk * 32), idS, kk > 0);
        mma_commit(&bars[LT_S]);
        if (!(ok = mbar_wait(&bars[LT_P], n & 1, abort, &g_fault_word))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma_bf16_ts(tO, tS + kk * 8, desc_add(dv, kk * 2048), idO, kk > 0);
        mma_commit(&bars[LT_T]);
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const float sc2 = g.lat_scale * kLog2e;
    uint4 pre_q[NQ];
    auto fetch = [&](int n) {
      const int r = (split + n * n_split) * BM + tid;
      const bool on = n < n_tiles && r < g.Tq;
      const uint4* qp = reinterpret_cast<const uint4*>(rq + ((int64_t)(b * g.Tq + (on ? r : 0)) * g.Lh + lh) * ldh);
#pragma unroll
      for (int i = 0; i < NQ; ++i) pre_q[i] = (on && 8 * i < ldh) ? __ldg(qp + i) : make_uint4(0, 0, 0, 0);
    };
    fetch(0);
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int r = (split + n * n_split) * BM + tid;
      const bool valid = r < g.Tq;
      const int qid = valid ? row_qid(g, r) : 0;
#pragma unroll
      for (int i = 0; i < NQ; ++i) *lat_chunk(smem + L::AQ, tid, i) = pre_q[i];
      fence_async_smem();
      mbar_arrive(&bars[LT_A]);
      fetch(n + 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[LT_S], n & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      float s[64];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(tS + lane_off, r0);
        tmem_ld32(tS + lane_off + 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = i < qid ? __uint_as_float(r0[i]) * sc2 : -INFINITY;
          s[32 + i] = 32 + i < qid ? __uint_as_float(r1[i]) * sc2 : -INFINITY;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 64; ++j) mx = fmaxf(mx, s[j]);
      const float mb = qid > 0 ? mx : 0.f;
      float l = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = 2 * i < qid ? fast_exp2(s[2 * i] - mb) : 0.f;
        const float p1 = 2 * i + 1 < qid ? fast_exp2(s[2 * i + 1] - mb) : 0.f;
        l += p0 + p1;
        pk[i] = pack_bf16(p0, p1);
      }
      {
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          lo[i] = pk[i];
          hi[i] = pk[16 + i];
        }
        tmem_st16(tS + lane_off, lo);
        tmem_st16(tS + lane_off + 16, hi);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars[LT_P]);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[LT_T], n & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      const float inv = qid > 0 ? 1.f / l : 0.f;
#pragma unroll
      for (int hh = 0; hh < LDH / 32; ++hh) {
        uint32_t o[32];
        tmem_ld32(tO + lane_off + hh * 32, o);
        tmem_ld_wait();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(lat + (int64_t)(b * g.Tq + r) * g.Ld + lh * ldh + hh * 32);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (hh * 32 + 8 * c < ldh)
              dst[c] = make_uint4(pack_bf16(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                                  pack_bf16(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                                  pack_bf16(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                                  pack_bf16(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
        }
      }
      if (valid) lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r] = qid > 0 ? (mb + log2f(l)) * kLn2 : INFINITY;
    }
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// Forward of the latent branch on the tensor cores for 64 < Nc <= 512 chunks
// (bf16, latent head dim <= 64 as above). All of (b, head)'s chunk keys and
// values sit in shared memory (128-byte rows, 64 KB each at 512 chunks). Per
// 128-row tile with nkt = ceil(qid(last row) / 64) key tiles, two passes over
// the key tiles, each tile S = rq gk^T (M128 x N64, bf16, fp32 accumulation)
// in one of two TMEM buffers so that the next tile's MMA overlaps this
// tile's softmax:
//   pass 1: the row max of the masked S sc (chunks j < qid(r));
//   pass 2: P = 2^(S sc - max) (masked, fp32; l sums it), P as bf16 over the
//           S columns, O += P gv_tile (A from TMEM) accumulated in TMEM.
// lat = O / l, lat_lse = max + ln l; rows that see no chunk write 0 and
// INFINITY (models.py:366-373). Recomputing S costs one small MMA per tile
// and keeps P exactly the fp32 value the normaliser sums, as in the 64-chunk
// kernel.
struct LatFwdLongLayout {
  static constexpr int AQ = 0;  // rq bf16 [128 rows][<= 64] in 128-byte rows
  static constexpr int GK = 16384;
  __host__ __device__ static constexpr int nc_pad(int nc) { return (nc + 63) / 64 * 64; }
  __host__ __device__ static constexpr int gv(int nc) { return GK + nc_pad(nc) * 128; }
  __host__ __device__ static constexpr int bar(int nc) { return GK + 2 * nc_pad(nc) * 128; }
  __host__ __device__ static constexpr int bytes(int nc) { return bar(nc) + 128; }
};
enum { LL_A = 0, LL_S = 1, LL_F = 3, LL_O = 5, LL_NB = 6 };

template <int LDH>
__global__ void __launch_bounds__(160, 1)
    latent_fwd_tc_long_kernel(Geom g, const bf16* __restrict__ rq, const bf16* __restrict__ gkv,
                              bf16* __restrict__ lat, float* __restrict__ lat_lse, int n_split) {
  using L = LatFwdLongLayout;
  constexpr int NQ = LDH / 8;
  extern __shared__ __align__(1024) uint8_t smem_latl_tc[];
  uint8_t* smem = smem_latl_tc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bar(g.Nc));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + LL_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int split = blockIdx.x, lh = blockIdx.y, b = blockIdx.z;
  const int n_rb = cdiv(g.Tq, BM);
  const int n_tiles = split < n_rb ? (n_rb - 1 - split) / n_split + 1 : 0;
  const int ldh = g.ldh;
  const int nc_pad = L::nc_pad(g.Nc);
  uint8_t* sgk = smem + L::GK;
  uint8_t* sgv = smem + L::gv(g.Nc);
  // key tiles a row tile needs: the chunks its last row sees
  auto tile_nkt = [&](int n) {
    const int rlast = min((split + n * n_split) * BM + BM - 1, g.Tq - 1);
    return cdiv(row_qid(g, rlast), 64);
  };

  if (tid == 0) {
    mbar_init(&bars[LL_A], BM);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[LL_S + s], 1);
      mbar_init(&bars[LL_F + s], BM);
    }
    mbar_init(&bars[LL_O], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    __syncwarp();
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  // chunk keys / values of (b, lh), 16-byte chunk (key, c); zero past Nc / ldh
  for (int idx = tid; idx < nc_pad * 8; idx += blockDim.x) {
    const int key = idx >> 3, c = idx & 7;
    const bool on = key < g.Nc && 8 * c < ldh;
    const int64_t base = ((int64_t)(b * g.Nc + (on ? key : 0)) * 2 * g.Lh + lh) * ldh;
    *lat_chunk(sgk, key, c) = on ? reinterpret_cast<const uint4*>(gkv + base)[c] : make_uint4(0, 0, 0, 0);
    *lat_chunk(sgv, key, c) =
        on ? reinterpret_cast<const uint4*>(gkv + base + (int64_t)g.Lh * ldh)[c] : make_uint4(0, 0, 0, 0);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 128;  // S buffers at [0,64) and [64,128) (P bf16 over the first 32 of each)

  if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, 64, false, false);  // rq gk^T
      constexpr uint32_t idO = idesc_bf16_f32(BM, 64, false, true);   // P gv
      const uint64_t daq = desc_sw128(smem_u32(smem + L::AQ), 16, 1024);
      const uint64_t dk = desc_sw128(smem_u32(sgk), 16, 1024);
      const uint64_t dv = desc_sw128(smem_u32(sgv), 8192, 1024);
      bool ok = true;
      int it = 0, no = 0;  // items (S tiles) issued so far, tiles with an O
      // S of item q (key tile kt) into buffer q&1, once item q-2 has left it
      auto issue_s = [&](int q, int kt) -> bool {
        if (q >= 2 && !mbar_wait(&bars[LL_F + (q & 1)], ((q - 2) >> 1) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint32_t tS = tmem + (q & 1) * 64;
#pragma unroll
        for (int kk = 0; kk < LDH / 16; ++kk)
          mma_bf16(tS, desc_add(daq, kk * 32), desc_add(dk, kt * 8192 + kk * 32), idS, kk > 0);
        mma_commit(&bars[LL_S + (q & 1)]);
        return true;
      };
      for (int n = 0; ok && n < n_tiles; ++n) {
        // the rows are staged (and the previous tile's O has been read)
        if (!(ok = mbar_wait(&bars[LL_A], n & 1, abort, &g_fault_word))) break;
        const int nkt = tile_nkt(n), N = 2 * nkt;
        if (N == 0) continue;
        if (!(ok = issue_s(it, 0))) break;
        for (int i = 0; ok && i < N; ++i) {
          const int q = it + i;
          if (i + 1 < N && !(ok = issue_s(q + 1, (i + 1) % nkt))) break;
          if (i >= nkt) {  // pass 2: P of item q written -> O += P gv
            if (!(ok = mbar_wait(&bars[LL_F + (q & 1)], (q >> 1) & 1, abort, &g_fault_word))) break;
            tc_fence_after();
            const int kt = i - nkt;
            const uint32_t tP = tmem + (q & 1) * 64;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ts(tO, tP + kk * 8, desc_add(dv, kt * 8192 + kk * 2048), idO, (i > nkt || kk > 0) ? 1u : 0u);
          }
        }
        if (!ok) break;
        mma_commit(&bars[LL_O]);
        it += N;
        ++no;
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const float sc2 = g.lat_scale * kLog2e;
    uint4 pre_q[NQ];
    auto fetch = [&](int n) {
      const int r = (split + n * n_split) * BM + tid;
      const bool on = n < n_tiles && r < g.Tq;
      const uint4* qp = reinterpret_cast<const uint4*>(rq + ((int64_t)(b * g.Tq + (on ? r : 0)) * g.Lh + lh) * ldh);
#pragma unroll
      for (int i = 0; i < NQ; ++i) pre_q[i] = (on && 8 * i < ldh) ? __ldg(qp + i) : make_uint4(0, 0, 0, 0);
    };
    fetch(0);
    bool ok = true;
    int it = 0, no = 0;
    for (int n = 0; n < n_tiles; ++n) {
      const int r = (split + n * n_split) * BM + tid;
      const bool valid = r < g.Tq;
      const int qid = valid ? row_qid(g, r) : 0;
#pragma unroll
      for (int i = 0; i < NQ; ++i) *lat_chunk(smem + L::AQ, tid, i) = pre_q[i];
      fence_async_smem();
      mbar_arrive(&bars[LL_A]);
      fetch(n + 1);
      const int nkt = tile_nkt(n), N = 2 * nkt;
      float m = -INFINITY, mb = 0.f, l = 0.f;
      for (int i = 0; i < N; ++i) {
        const int q = it + i, kt = i < nkt ? i : i - nkt;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[LL_S + (q & 1)], (q >> 1) & 1, abort, &g_fault_word));
        if (!ok) break;
        tc_fence_after();
        const uint32_t tS = tmem + lane_off + (q & 1) * 64;
        uint32_t r0[32], r1[32];
        tmem_ld32(tS, r0);
        tmem_ld32(tS + 32, r1);
        tmem_ld_wait();
        const int c_hi = qid - kt * 64;  // columns c < c_hi are visible
        if (i < nkt) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            if (c < c_hi) m = fmaxf(m, __uint_as_float(r0[c]) * sc2);
            if (32 + c < c_hi) m = fmaxf(m, __uint_as_float(r1[c]) * sc2);
          }
        } else {
          if (i == nkt) mb = qid > 0 ? m : 0.f;
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float p0 = 2 * c < c_hi ? fast_exp2(__uint_as_float(r0[2 * c]) * sc2 - mb) : 0.f;
            const float p1 = 2 * c + 1 < c_hi ? fast_exp2(__uint_as_float(r0[2 * c + 1]) * sc2 - mb) : 0.f;
            const float p2 = 32 + 2 * c < c_hi ? fast_exp2(__uint_as_float(r1[2 * c]) * sc2 - mb) : 0.f;
            const float p3 = 33 + 2 * c < c_hi ? fast_exp2(__uint_as_float(r1[2 * c + 1]) * sc2 - mb) : 0.f;
            l += (p0 + p1) + (p2 + p3);
            lo[c] = pack_bf16(p0, p1);
            hi[c] = pack_bf16(p2, p3);
          }
          tmem_st16(tS, lo);
          tmem_st16(tS + 16, hi);
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(&bars[LL_F + (q & 1)]);
      }
      if (!ok) break;
      it += N;
      const float inv = qid > 0 ? 1.f / l : 0.f;
      if (N > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[LL_O], no & 1, abort, &g_fault_word));
        if (!ok) break;
        ++no;
        tc_fence_after();
      }
#pragma unroll
      for (int hh = 0; hh < LDH / 32; ++hh) {
        uint32_t o[32];
        if (N > 0) {
          tmem_ld32(tO + lane_off + hh * 32, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(lat + (int64_t)(b * g.Tq + r) * g.Ld + lh * ldh + hh * 32);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (hh * 32 + 8 * c < ldh)
              dst[c] = make_uint4(pack_bf16(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                                  pack_bf16(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                                  pack_bf16(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                                  pack_bf16(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
        }
      }
      // O has been read: the next tile's first P gv may overwrite it (the
      // MMA thread waits for LL_A, which these threads arrive on next)
      tc_fence_before();
      if (valid) lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r] = qid > 0 ? (mb + log2f(l)) * kLn2 : INFINITY;
    }
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// Backward of the latent branch on the tensor cores for 64 < Nc <= 512 (bf16,
// latent head dim <= 64). With P = softmax over visible chunks, dP = dlat gv,
// delta = sum_j P dP, dS = P (dP - delta):
//   drq = lat_scale dS gk,  dgk = lat_scale dS^T rq,  dgv = P^T dlat.
// Two kernels:
//   rows: per 128-row tile, two passes over 64-key tiles (pass 1 sums delta
//         in fp32, pass 2 forms dS and accumulates drq = dS gk in TMEM);
//         writes drq and delta (for the key kernel);
//   keys: per 128-key tile, 64-row steps: S^T, dP^T recomputed, P^T / dS^T
//         in TMEM, dgk += dS^T rq and dgv += P^T dlat accumulated in TMEM;
//         one partial per row split ([split][b][key][2][Ld], the SIMT
//         kernel's layout, summed by the reduce kernel).
// dP is two bf16 MMAs, dlat = hi + lo (both bf16) against gv: ~16 mantissa
// bits, since dP - delta cancels when the pooled values are close. S uses
// the bf16 rq / gk the forward used, so P matches the saved lse.
struct LatBwdRowsLayout {
  static constexpr int AQ = 0;        // rq bf16 [128 rows][<= 64] in 128-byte rows
  static constexpr int DH = 16384;    // dlat hi bf16 [128][<= 64]
  static constexpr int DL = 32768;    // dlat lo bf16
  static constexpr int GK = 49152;    // gk bf16 [Nc_pad][<= 64]
  __host__ __device__ static constexpr int nc_pad(int nc) { return (nc + 63) / 64 * 64; }
  __host__ __device__ static constexpr int gv(int nc) { return GK + nc_pad(nc) * 128; }
  __host__ __device__ static constexpr int bar(int nc) { return GK + 2 * nc_pad(nc) * 128; }
  __host__ __device__ static constexpr int bytes(int nc) { return bar(nc) + 128; }
};

// dlat row (fp32, 4 per 16-byte chunk) -> hi / lo bf16 16-byte chunks c
__device__ __forceinline__ void split_hi_lo(const float4 a, const float4 b, uint4& hi, uint4& lo) {
  const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t hp = pack_bf16(x[2 * i], x[2 * i + 1]);
    const float h0 = __uint_as_float(hp << 16), h1 = __uint_as_float(hp & 0xffff0000u);
    h[i] = hp;
    l[i] = pack_bf16(x[2 * i] - h0, x[2 * i + 1] - h1);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int LDH>
__global__ void __launch_bounds__(160, 1)
    latent_bwd_rows_tc_kernel(Geom g, const bf16* __restrict__ rq, const bf16* __restrict__ gkv,
                              const float* __restrict__ lat_lse, const float* __restrict__ dlat,
                              bf16* __restrict__ drq, float* __restrict__ delta_out, int n_split) {
  using L = LatBwdRowsLayout;
  constexpr int NQ = LDH / 8;
  extern __shared__ __align__(1024) uint8_t smem_latbr_tc[];
  uint8_t* smem = smem_latbr_tc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bar(g.Nc));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + LL_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int split = blockIdx.x, lh = blockIdx.y, b = blockIdx.z;
  const int n_rb = cdiv(g.Tq, BM);
  const int n_tiles = split < n_rb ? (n_rb - 1 - split) / n_split + 1 : 0;
  const int ldh = g.ldh;
  const int nc_pad = L::nc_pad(g.Nc);
  uint8_t* sgk = smem + L::GK;
  uint8_t* sgv = smem + L::gv(g.Nc);
  auto tile_nkt = [&](int n) {
    const int rlast = min((split + n * n_split) * BM + BM - 1, g.Tq - 1);
    return cdiv(row_qid(g, rlast), 64);
  };

  if (tid == 0) {
    mbar_init(&bars[LL_A], BM);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[LL_S + s], 1);
      mbar_init(&bars[LL_F + s], BM);
    }
    mbar_init(&bars[LL_O], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    __syncwarp();
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  for (int idx = tid; idx < nc_pad * 8; idx += blockDim.x) {
    const int key = idx >> 3, c = idx & 7;
    const bool on = key < g.Nc && 8 * c < ldh;
    const int64_t base = ((int64_t)(b * g.Nc + (on ? key : 0)) * 2 * g.Lh + lh) * ldh;
    *lat_chunk(sgk, key, c) = on ? reinterpret_cast<const uint4*>(gkv + base)[c] : make_uint4(0, 0, 0, 0);
    *lat_chunk(sgv, key, c) =
        on ? reinterpret_cast<const uint4*>(gkv + base + (int64_t)g.Lh * ldh)[c] : make_uint4(0, 0, 0, 0);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // buffer q&1: S at (q&1)*128 (dS bf16 over its first 32 columns), dP 64 on;
  // drq accumulator at 256
  const uint32_t tQ = tmem + 256;

  if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, 64, false, false);  // rq gk^T, dlat gv^T
      constexpr uint32_t idQ = idesc_bf16_f32(BM, 64, false, true);   // dS gk
      const uint64_t daq = desc_sw128(smem_u32(smem + L::AQ), 16, 1024);
      const uint64_t ddh = desc_sw128(smem_u32(smem + L::DH), 16, 1024);
      const uint64_t ddl = desc_sw128(smem_u32(smem + L::DL), 16, 1024);
      const uint64_t dk = desc_sw128(smem_u32(sgk), 16, 1024);
      const uint64_t dv = desc_sw128(smem_u32(sgv), 16, 1024);
      const uint64_t dkm = desc_sw128(smem_u32(sgk), 8192, 1024);
      bool ok = true;
      int it = 0;
      auto issue_sp = [&](int q, int kt) -> bool {
        if (q >= 2 && !mbar_wait(&bars[LL_F + (q & 1)], ((q - 2) >> 1) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint32_t tS = tmem + (q & 1) * 128, tP = tS + 64;
#pragma unroll
        for (int kk = 0; kk < LDH / 16; ++kk) {
          const uint32_t bo = kt * 8192 + kk * 32;
          mma_bf16(tS, desc_add(daq, kk * 32), desc_add(dk, bo), idS, kk > 0);
          mma_bf16(tP, desc_add(ddh, kk * 32), desc_add(dv, bo), idS, kk > 0);
          mma_bf16(tP, desc_add(ddl, kk * 32), desc_add(dv, bo), idS, 1u);
        }
        mma_commit(&bars[LL_S + (q & 1)]);
        return true;
      };
      for (int n = 0; ok && n < n_tiles; ++n) {
        if (!(ok = mbar_wait(&bars[LL_A], n & 1, abort, &g_fault_word))) break;
        const int nkt = tile_nkt(n), N = 2 * nkt;
        if (N == 0) continue;
        if (!(ok = issue_sp(it, 0))) break;
        for (int i = 0; ok && i < N; ++i) {
          const int q = it + i;
          if (i + 1 < N && !(ok = issue_sp(q + 1, (i + 1) % nkt))) break;
          if (i >= nkt) {  // pass 2: dS of item q written -> drq += dS gk
            if (!(ok = mbar_wait(&bars[LL_F + (q & 1)], (q >> 1) & 1, abort, &g_fault_word))) break;
            tc_fence_after();
            const int kt = i - nkt;
            const uint32_t tA = tmem + (q & 1) * 128;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ts(tQ, tA + kk * 8, desc_add(dkm, kt * 8192 + kk * 2048), idQ, (i > nkt || kk > 0) ? 1u : 0u);
          }
        }
        if (!ok) break;
        mma_commit(&bars[LL_O]);
        it += N;
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const float sc2 = g.lat_scale * kLog2e;
    bool ok = true;
    int it = 0, no = 0;
    for (int n = 0; n < n_tiles; ++n) {
      const int r = (split + n * n_split) * BM + tid;
      const bool valid = r < g.Tq;
      const int qid = valid ? row_qid(g, r) : 0;
      const float lse2 = valid ? lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r] * kLog2e : INFINITY;
      {  // this row's rq and dlat (hi / lo) into the operand tiles
        const uint4* qp = reinterpret_cast<const uint4*>(rq + ((int64_t)(b * g.Tq + (valid ? r : 0)) * g.Lh + lh) * ldh);
        const float4* dp = reinterpret_cast<const float4*>(dlat + (int64_t)(b * g.Tq + (valid ? r : 0)) * g.Ld + lh * ldh);
#pragma unroll
        for (int i = 0; i < NQ; ++i) {
          const bool on = valid && 8 * i < ldh;
          *lat_chunk(smem + L::AQ, tid, i) = on ? __ldg(qp + i) : make_uint4(0, 0, 0, 0);
          uint4 hi = make_uint4(0, 0, 0, 0), lo = hi;
          if (on) split_hi_lo(__ldg(dp + 2 * i), __ldg(dp + 2 * i + 1), hi, lo);
          *lat_chunk(smem + L::DH, tid, i) = hi;
          *lat_chunk(smem + L::DL, tid, i) = lo;
        }
      }
      fence_async_smem();
      mbar_arrive(&bars[LL_A]);
      const int nkt = tile_nkt(n), N = 2 * nkt;
      float delta = 0.f;
      for (int i = 0; i < N; ++i) {
        const int q = it + i, kt = i < nkt ? i : i - nkt;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[LL_S + (q & 1)], (q >> 1) & 1, abort, &g_fault_word));
        if (!ok) break;
        tc_fence_after();
        const uint32_t tS = tmem + lane_off + (q & 1) * 128, tP = tS + 64;
        const int c_hi = qid - kt * 64;  // columns c < c_hi are visible
        uint32_t pk[32];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t rs[32], rp[32];
          tmem_ld32(tS + hh * 32, rs);
          tmem_ld32(tP + hh * 32, rp);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const int j = hh * 32 + c;
            const float p0 = j < c_hi ? fast_exp2(fmaf(__uint_as_float(rs[c]), sc2, -lse2)) : 0.f;
            const float p1 = j + 1 < c_hi ? fast_exp2(fmaf(__uint_as_float(rs[c + 1]), sc2, -lse2)) : 0.f;
            const float d0 = __uint_as_float(rp[c]), d1 = __uint_as_float(rp[c + 1]);
            if (i < nkt) {
              delta = fmaf(p0, d0, delta);
              delta = fmaf(p1, d1, delta);
            } else {
              pk[hh * 16 + c / 2] = pack_bf16(p0 * (d0 - delta), p1 * (d1 - delta));
            }
          }
        }
        if (i >= nkt) {
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            lo[c] = pk[c];
            hi[c] = pk[16 + c];
          }
          tmem_st16(tS, lo);
          tmem_st16(tS + 16, hi);
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(&bars[LL_F + (q & 1)]);
      }
      if (!ok) break;
      it += N;
      if (N > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[LL_O], no & 1, abort, &g_fault_word));
        if (!ok) break;
        ++no;
        tc_fence_after();
      }
#pragma unroll
      for (int hh = 0; hh < LDH / 32; ++hh) {
        uint32_t o[32];
        if (N > 0) {
          tmem_ld32(tQ + lane_off + hh * 32, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
        if (valid) {
          const float s = g.lat_scale;
          uint4* dst = reinterpret_cast<uint4*>(drq + ((int64_t)(b * g.Tq + r) * g.Lh + lh) * ldh + hh * 32);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (hh * 32 + 8 * c < ldh)
              dst[c] = make_uint4(pack_bf16(__uint_as_float(o[8 * c]) * s, __uint_as_float(o[8 * c + 1]) * s),
                                  pack_bf16(__uint_as_float(o[8 * c + 2]) * s, __uint_as_float(o[8 * c + 3]) * s),
                                  pack_bf16(__uint_as_float(o[8 * c + 4]) * s, __uint_as_float(o[8 * c + 5]) * s),
                                  pack_bf16(__uint_as_float(o[8 * c + 6]) * s, __uint_as_float(o[8 * c + 7]) * s));
        }
      }
      // drq has been read and the tile's MMAs are done with the operand
      // tiles: the next tile may overwrite both
      tc_fence_before();
      if (valid) delta_out[(int64_t)(b * g.Lh + lh) * g.Tq + r] = delta;
    }
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// keys kernel: CTA = (128-key tile kt2 and row split rs, latent head, b).
// Its row steps (64 rows each) are those holding a row that sees a key of
// the tile (rows r with qid(r) > k0, a suffix of the rows), every n_split-th
// from its first. Per step, double-buffered in shared memory (staged by the
// key threads, two threads per row) and TMEM:
//   S^T = gk rq^T, dP^T = gv (dlat_hi + dlat_lo)^T   (M128 keys x N64 rows)
//   P^T = 2^(S^T sc - lse2[row]) on visible (key j < qid(row)), dS^T =
//   P^T (dP^T - delta[row]), both bf16 over the first 32 columns of their
//   buffers; dgk += dS^T rq, dgv += P^T dlat_hi (A from TMEM, N = 64).
struct LatBwdKeysLayout {
  static constexpr int GKA = 0;               // gk bf16 [128 keys][<= 64]
  static constexpr int GVA = 16384;           // gv bf16 [128 keys][<= 64]
  static constexpr int STEP = 32768;          // per buffer: rq, dlat hi, dlat lo [64 rows][<= 64] bf16
  static constexpr int STEP_BYTES = 3 * 8192;
  static constexpr int VEC = STEP + 2 * STEP_BYTES;  // per buffer: lse2[64], delta[64], qid[64]
  static constexpr int BAR = VEC + 2 * 3 * 64 * 4;
  static constexpr int BYTES = BAR + 256;
  // shared memory asked for at launch: enough that one CTA (512 TMEM columns) holds an SM
  static constexpr int LAUNCH = 120 * 1024;
};
enum { LK_A = 0, LK_S = 2, LK_F = 4, LK_E = 6, LK_O = 8, LK_NB = 9 };

template <int LDH>
__global__ void __launch_bounds__(160, 1)
    latent_bwd_keys_tc_kernel(Geom g, const bf16* __restrict__ rq, const bf16* __restrict__ gkv,
                              const float* __restrict__ lat_lse, const float* __restrict__ dlat,
                              const float* __restrict__ delta, float* __restrict__ part, int n_split) {
  using L = LatBwdKeysLayout;
  extern __shared__ __align__(1024) uint8_t smem_latbk_tc[];
  uint8_t* smem = smem_latbk_tc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + LK_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int kt2 = blockIdx.x / n_split, rs = blockIdx.x % n_split, lh = blockIdx.y, b = blockIdx.z;
  const int k0 = kt2 * BM, ldh = g.ldh;
  // first row that sees key k0: off + r qbs >= (k0 + 1) cs (and k0 < Nc - 1:
  // qid never exceeds Nc - 1, so the last chunk is seen by no row)
  int r_first = g.Tq;
  if (k0 < g.Nc - 1) {
    const int need = (k0 + 1) * g.cs - g.off;
    r_first = need <= 0 ? 0 : min(g.Tq, (need + g.qbs - 1) / g.qbs);
  }
  const int s_first = r_first / 64, n_steps_all = cdiv(g.Tq, 64);
  const int n_steps = s_first + rs < n_steps_all ? (n_steps_all - 1 - s_first - rs) / n_split + 1 : 0;
  auto step_row0 = [&](int i) { return (s_first + rs + i * n_split) * 64; };

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[LK_A + s], BM);
      mbar_init(&bars[LK_S + s], 1);
      mbar_init(&bars[LK_F + s], BM);
      mbar_init(&bars[LK_E + s], 1);
    }
    mbar_init(&bars[LK_O], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    __syncwarp();
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // the key tile's gk / gv rows (A operands), zero past Nc / ldh
  for (int idx = tid; idx < BM * 8; idx += blockDim.x) {
    const int kr = idx >> 3, c = idx & 7, key = k0 + kr;
    const bool on = key < g.Nc && 8 * c < ldh;
    const int64_t base = ((int64_t)(b * g.Nc + (on ? key : 0)) * 2 * g.Lh + lh) * ldh;
    *lat_chunk(smem + L::GKA, kr, c) = on ? reinterpret_cast<const uint4*>(gkv + base)[c] : make_uint4(0, 0, 0, 0);
    *lat_chunk(smem + L::GVA, kr, c) =
        on ? reinterpret_cast<const uint4*>(gkv + base + (int64_t)g.Lh * ldh)[c] : make_uint4(0, 0, 0, 0);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // buffer i&1: S^T at (i&1)*128 (P^T bf16 over its first 32 columns), dP^T
  // 64 on (dS^T bf16 over its first 32); dgk at 256, dgv at 320
  const uint32_t tGK = tmem + 256, tGV = tmem + 320;

  if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, 64, false, false);  // gk rq^T, gv dlat^T
      constexpr uint32_t idG = idesc_bf16_f32(BM, 64, false, true);   // dS^T rq, P^T dlat
      const uint64_t dka = desc_sw128(smem_u32(smem + L::GKA), 16, 1024);
      const uint64_t dva = desc_sw128(smem_u32(smem + L::GVA), 16, 1024);
      bool ok = true;
      for (int i = 0; ok && i < n_steps; ++i) {
        const int s = i & 1;
        uint8_t* st = smem + L::STEP + s * L::STEP_BYTES;
        // rows staged; TMEM buffer s free (step i-2's P^T / dS^T consumed by
        // its dgk / dgv MMAs, issued before this in pipe order)
        if (!(ok = mbar_wait(&bars[LK_A + s], (i >> 1) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint64_t dq = desc_sw128(smem_u32(st), 16, 1024);
        const uint64_t ddh = desc_sw128(smem_u32(st + 8192), 16, 1024);
        const uint64_t ddl = desc_sw128(smem_u32(st + 16384), 16, 1024);
        const uint32_t tS = tmem + s * 128, tP = tS + 64;
#pragma unroll
        for (int kk = 0; kk < LDH / 16; ++kk) {
          mma_bf16(tS, desc_add(dka, kk * 32), desc_add(dq, kk * 32), idS, kk > 0);
          mma_bf16(tP, desc_add(dva, kk * 32), desc_add(ddh, kk * 32), idS, kk > 0);
          mma_bf16(tP, desc_add(dva, kk * 32), desc_add(ddl, kk * 32), idS, 1u);
        }
        mma_commit(&bars[LK_S + s]);
        if (!(ok = mbar_wait(&bars[LK_F + s], (i >> 1) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint64_t dqm = desc_sw128(smem_u32(st), 8192, 1024);
        const uint64_t ddm = desc_sw128(smem_u32(st + 8192), 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16_ts(tGK, tP + kk * 8, desc_add(dqm, kk * 2048), idG, (i > 0 || kk > 0) ? 1u : 0u);
          mma_bf16_ts(tGV, tS + kk * 8, desc_add(ddm, kk * 2048), idG, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars[LK_E + s]);  // the step's rows may be restaged
      }
      if (ok) mma_commit(&bars[LK_O]);
      else raise_fault(g, kFaultMma, abort);
    }
  } else {
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const float sc2 = g.lat_scale * kLog2e;
    const int key = k0 + tid;  // this thread's TMEM lane
    // stage step i's rows into buffer i&1: two threads per row (half the row's chunks each)
    auto stage = [&](int i) {
      const int s = i & 1, row = tid >> 1, h = tid & 1;
      const int r = step_row0(i) + row;
      const bool valid = r < g.Tq;
      uint8_t* st = smem + L::STEP + s * L::STEP_BYTES;
      const uint4* qp = reinterpret_cast<const uint4*>(rq + ((int64_t)(b * g.Tq + (valid ? r : 0)) * g.Lh + lh) * ldh);
      const float4* dp = reinterpret_cast<const float4*>(dlat + (int64_t)(b * g.Tq + (valid ? r : 0)) * g.Ld + lh * ldh);
#pragma unroll
      for (int c = h * 4; c < h * 4 + 4; ++c) {
        const bool on = valid && 8 * c < ldh;
        uint4 hi = make_uint4(0, 0, 0, 0), lo = hi;
        if (on) split_hi_lo(__ldg(dp + 2 * c), __ldg(dp + 2 * c + 1), hi, lo);
        *lat_chunk(st, row, c) = on ? __ldg(qp + c) : make_uint4(0, 0, 0, 0);
        *lat_chunk(st + 8192, row, c) = hi;
        *lat_chunk(st + 16384, row, c) = lo;
      }
      float* v = reinterpret_cast<float*>(smem + L::VEC) + s * 192;
      if (h == 0) {
        v[row] = valid ? lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r] * kLog2e : INFINITY;
        v[64 + row] = valid ? delta[(int64_t)(b * g.Lh + lh) * g.Tq + r] : 0.f;
        reinterpret_cast<int*>(v)[128 + row] = valid ? row_qid(g, r) : 0;
      }
      fence_async_smem();
      mbar_arrive(&bars[LK_A + s]);
    };
    bool ok = true;
    if (n_steps > 0) stage(0);
    for (int i = 0; i < n_steps; ++i) {
      const int s = i & 1;
      if (i + 1 < n_steps) {
        // buffer (i+1)&1 held step i-1: its dgk / dgv MMAs must be done
        if (i >= 1) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bars[LK_E + ((i + 1) & 1)], ((i - 1) >> 1) & 1, abort,
                                                 &g_fault_word));
          if (!ok) break;
        }
        stage(i + 1);
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[LK_S + s], (i >> 1) & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      const float* v = reinterpret_cast<const float*>(smem + L::VEC) + s * 192;
      const int* vq = reinterpret_cast<const int*>(v) + 128;
      const uint32_t tS = tmem + lane_off + s * 128, tP = tS + 64;
      uint32_t pp[32], pd[32];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t rs_[32], rp[32];
        tmem_ld32(tS + hh * 32, rs_);
        tmem_ld32(tP + hh * 32, rp);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const int col = hh * 32 + c;
          const float p0 = key < vq[col] ? fast_exp2(fmaf(__uint_as_float(rs_[c]), sc2, -v[col])) : 0.f;
          const float p1 = key < vq[col + 1] ? fast_exp2(fmaf(__uint_as_float(rs_[c + 1]), sc2, -v[col + 1])) : 0.f;
          pp[hh * 16 + c / 2] = pack_bf16(p0, p1);
          pd[hh * 16 + c / 2] = pack_bf16(p0 * (__uint_as_float(rp[c]) - v[64 + col]),
                                          p1 * (__uint_as_float(rp[c + 1]) - v[64 + col + 1]));
        }
      }
      {
        uint32_t a[16], c2[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          a[c] = pp[c];
          c2[c] = pp[16 + c];
        }
        tmem_st16(tS, a);
        tmem_st16(tS + 16, c2);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          a[c] = pd[c];
          c2[c] = pd[16 + c];
        }
        tmem_st16(tP, a);
        tmem_st16(tP + 16, c2);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars[LK_F + s]);
    }
    if (ok && n_steps > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars[LK_O], 0, abort, &g_fault_word));
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
    // this CTA's partial: [rs][b][key][2][Ld] at lh * ldh + e. The TMEM loads
    // are warp-collective: every lane loads, lanes past Nc store nothing.
    tc_fence_after();
    {
      float* my_part = part + (((int64_t)rs * g.B + b) * g.Nc + (key < g.Nc ? key : 0)) * 2 * g.Ld + lh * ldh;
      const bool have = __all_sync(0xffffffffu, ok && n_steps > 0 && !*abort);
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const float mul = which == 0 ? g.lat_scale : 1.f;
#pragma unroll
        for (int hh = 0; hh < LDH / 32; ++hh) {
          uint32_t o[32];
          if (have) {
            tmem_ld32((which == 0 ? tGK : tGV) + lane_off + hh * 32, o);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = 0u;
          }
          if (key < g.Nc) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (hh * 32 + c < ldh) my_part[(int64_t)which * g.Ld + hh * 32 + c] = __uint_as_float(o[c]) * mul;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
