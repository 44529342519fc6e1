// Backward of the tensor-core local branch (included by local_sm100.cu, which
// provides the fault word, the tensor-map helpers and the ptx wrappers).
//
// With s = scale q.k, P = exp(s - lse) on visible pairs, dO = dlocal (the
// gate backward's gradient of the local output), D = rowsum(dO * O):
//   dS = P (dO.v - D),  dq = scale sum_j dS k_j,  dk_j = scale sum_t dS q_t,
//   dv_j = sum_t P dO_t.
// Two kernels, no atomics, deterministic:
//   dq  : persistent, units of (b, h, 128-query tile); loops over 64-key tiles.
//   dkv : persistent, units of (b, h, 128-key tile); loops over 64-query
//         tiles t in [k0+1, k0+127+W].
// Both keep the two score-like tiles (S and dP) of the current inner tile in
// TMEM, double-buffered, so the softmax warps of tile j overlap the MMAs of
// tile j+1.

// ---------------------------------------------------------------------------
// dq, persistent: one CTA per SM walks the (h, query tile, b) units
// u = blockIdx.x + k * gridDim.x, heads fastest. Q/dO are double-buffered by
// unit (unit n uses buffer n&1), the K/V ring and the S/dP buffers run on
// counters that continue across units, so the next unit's Q/dO and first
// K/V tiles load and its first score MMAs run while this unit's dQ is read
// out of TMEM, staged over its own (no longer read) Q tile and stored.

template <int HD>
struct DqpLayout {
  static constexpr int BNK = 64;                   // keys per inner tile
  static constexpr int NKS = 3;                    // K / V stages
  static constexpr int QPANEL = BM * 128;          // 128-row panel (16 KB)
  static constexpr int KPANEL = BNK * 128;         // 64-row panel (8 KB)
  static constexpr int QTILE = BM * HD * 2;
  static constexpr int KTILE = BNK * HD * 2;
  static constexpr int QD = 2 * QTILE;             // one Q/dO buffer: Q (then dQ staging), dO
  static constexpr int Q = 0;                      // + qb * QD
  static constexpr int DO = QTILE;                 // + qb * QD
  static constexpr int K = 2 * QD;                 // NKS stages of K, V
  static constexpr int V = K + KTILE;
  static constexpr int KV = 2 * KTILE;             // bytes of one K/V stage
  static constexpr int BAR = K + NKS * KV;
  static constexpr int BYTES = BAR + 256;
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

// barriers: per Q/dO buffer loaded / free again (dQ store has read the
// staging); per K/V stage loaded / released; per TMEM buffer S,dP ready /
// dS written; dQ of a unit complete; dQ staged
enum {
  DP_Q = 0, DP_QE = 2, DP_KV = 4, DP_KVE = 7, DP_SP = 10, DP_DS = 12, DP_ACC = 14, DP_STG = 15, DP_NB = 16
};

struct DqUnit {
  int h, q0, b, kbase, nk;
};
template <int BNK>
__device__ __forceinline__ DqUnit dq_unit(const Geom& g, int u) {
  DqUnit t;
  const int nqt = cdiv(g.T, BM);
  t.h = u % g.H;
  const int r = u / g.H;
  t.q0 = (r % nqt) * BM;
  t.b = r / nqt;
  const int qlast = min(t.q0 + BM - 1, g.T - 1);
  t.kbase = local_lo(g, t.q0);
  const int khi = qlast - 1;
  t.nk = khi >= t.kbase ? (khi - t.kbase + BNK) / BNK : 0;
  return t;
}

template <int HD>
__global__ void __launch_bounds__(320, 1)
    local_dq_persist_kernel(const __grid_constant__ CUtensorMap tm_qkv128, const __grid_constant__ CUtensorMap tm_qkv64,
                            const __grid_constant__ CUtensorMap tm_do128, const __grid_constant__ CUtensorMap tm_st,
                            Geom g, const float* __restrict__ lse, const float* __restrict__ delta, int n_units) {
  using L = DqpLayout<HD>;
  constexpr int BNK = L::BNK, NKS = L::NKS;
  extern __shared__ __align__(1024) uint8_t smem_dqp[];
  uint8_t* smem = smem_dqp;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + DP_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {  // the swizzled layouts need 1024-byte alignment
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int qb = 0; qb < 2; ++qb) {
      mbar_init(&bars[DP_Q + qb], 1);
      mbar_init(&bars[DP_QE + qb], 1);
    }
    for (int s = 0; s < NKS; ++s) {
      mbar_init(&bars[DP_KV + s], 1);
      mbar_init(&bars[DP_KVE + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[DP_SP + s], 1);
      mbar_init(&bars[DP_DS + s], 2 * BM);
    }
    mbar_init(&bars[DP_ACC], 1);
    mbar_init(&bars[DP_STG], 2 * BM);
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
  // S buffers at columns [0,64) and [64,128); dP at [128,192) and [192,256);
  // dQ at [256, 256+HD). dS (bf16) is written back over the first 16 of each
  // 32 dP columns that produced it and feeds the dQ MMA from TMEM. One dQ
  // accumulator suffices: the first dQ MMA of a unit waits for that unit's
  // first dS, which the compute warps write only after reading out the
  // previous unit's dQ.
  const uint32_t tDQ = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_qkv128);
      prefetch_tmap(&tm_qkv64);
      prefetch_tmap(&tm_do128);
      prefetch_tmap(&tm_st);
      int jj = 0, n = 0, issued_kv = 0, issued_q = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++n) {
        const DqUnit t = dq_unit<BNK>(g, u);
        const int qb = n & 1;
        // buffer qb: free once unit n-2's dQ store has read its staging
        if (n >= 2 && !(ok = mbar_wait(&bars[DP_QE + qb], ((n >> 1) - 1) & 1, abort, &g_fault_word))) break;
        mbar_expect_tx(&bars[DP_Q + qb], 2 * L::QTILE);
        tma_load_tile<HD / 64, BM>(&tm_qkv128, &bars[DP_Q + qb], smem + qb * L::QD + L::Q, t.q0, t.h, t.b);
        tma_load_tile<HD / 64, BM>(&tm_do128, &bars[DP_Q + qb], smem + qb * L::QD + L::DO, t.q0, t.h, t.b);
        issued_q = n + 1;
        for (int j = 0; j < t.nk; ++j, ++jj) {
          const int s = jj % NKS;
          if (jj >= NKS && !(ok = mbar_wait(&bars[DP_KVE + s], ((jj / NKS) - 1) & 1, abort, &g_fault_word))) break;
          const int k0 = t.kbase + j * BNK;
          mbar_expect_tx(&bars[DP_KV + s], 2 * L::KTILE);
          tma_load_tile<HD / 64, 64>(&tm_qkv64, &bars[DP_KV + s], smem + L::K + s * L::KV, k0, g.H + t.h, t.b);
          tma_load_tile<HD / 64, 64>(&tm_qkv64, &bars[DP_KV + s], smem + L::V + s * L::KV, k0, 2 * g.H + t.h, t.b);
          issued_kv = jj + 1;
        }
      }
      if (!ok) {
        raise_fault(g, kFaultProducer, abort);
        // let the copies already issued land before the CTA can exit
        volatile int none = 0;
        volatile unsigned gnone = 0;
        for (int q = issued_q - 2 < 0 ? 0 : issued_q - 2; q < issued_q; ++q)
          mbar_wait(&bars[DP_Q + (q & 1)], (q >> 1) & 1, &none, &gnone, 100000000ull);
        for (int k = issued_kv - NKS < 0 ? 0 : issued_kv - NKS; k < issued_kv; ++k)
          mbar_wait(&bars[DP_KV + k % NKS], (k / NKS) & 1, &none, &gnone, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idSP = idesc_bf16_f32(BM, BNK, false, false);  // Q K^T, dO V^T
      constexpr uint32_t idDQ = idesc_bf16_f32(BM, HD, false, true);    // dS K (K MN-major)
      const uint64_t dq0 = desc_sw128(smem_u32(smem + L::Q), 16, 1024);
      const uint64_t ddo0 = desc_sw128(smem_u32(smem + L::DO), 16, 1024);
      const uint64_t dk0 = desc_sw128(smem_u32(smem + L::K), 16, 1024);
      const uint64_t dv0 = desc_sw128(smem_u32(smem + L::V), 16, 1024);
      const uint64_t dkm0 = desc_sw128(smem_u32(smem + L::K), L::KPANEL, 1024);
      // cursor over the (unit, key tile) items of this CTA, units without
      // keys skipped (n still counts them: it picks the Q/dO buffer)
      struct Cur {
        int u, n, j;
        DqUnit t;
      };
      auto skip_empty = [&](Cur& c) {
        while (c.u < n_units && c.t.nk == 0) {
          c.u += gridDim.x;
          ++c.n;
          if (c.u < n_units) c.t = dq_unit<BNK>(g, c.u);
        }
      };
      auto advance = [&](Cur& c) {
        if (++c.j < c.t.nk) return;
        c.j = 0;
        c.u += gridDim.x;
        ++c.n;
        if (c.u < n_units) c.t = dq_unit<BNK>(g, c.u);
        skip_empty(c);
      };
      auto issue_sp = [&](const Cur& c, int jj) -> bool {
        const int s = jj & 1, sk = jj % NKS, qb = c.n & 1;
        if (c.j == 0 && !mbar_wait(&bars[DP_Q + qb], (c.n >> 1) & 1, abort, &g_fault_word)) return false;
        if (!mbar_wait(&bars[DP_KV + sk], (jj / NKS) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint64_t dq = desc_add(dq0, qb * L::QD), ddo = desc_add(ddo0, qb * L::QD);
        const uint64_t dk = desc_add(dk0, sk * L::KV), dv = desc_add(dv0, sk * L::KV);
        const uint32_t tS = tmem + s * BNK, tP = tmem + 128 + s * BNK;
        // K steps past a padded head_dim would multiply zero-filled columns: skipped
#pragma unroll
        for (int kk = 0; kk < HD / 16 && kk * 16 < g.hd; ++kk) {
          const uint32_t aoff = (kk / 4) * L::QPANEL + (kk % 4) * 32;
          const uint32_t boff = (kk / 4) * L::KPANEL + (kk % 4) * 32;
          mma_bf16(tS, desc_add(dq, aoff), desc_add(dk, boff), idSP, kk > 0);
          mma_bf16(tP, desc_add(ddo, aoff), desc_add(dv, boff), idSP, kk > 0);
        }
        mma_commit(&bars[DP_SP + s]);
        return true;
      };
      Cur cur;
      cur.u = blockIdx.x;
      cur.n = 0;
      cur.j = 0;
      if (cur.u < n_units) cur.t = dq_unit<BNK>(g, cur.u);
      skip_empty(cur);
      bool ok = true;
      int jj = 0;
      if (cur.u < n_units) ok = issue_sp(cur, 0);
      // S/dP of the next item are issued before dQ of this one: the compute
      // warps wait for them next, and they may start once dQ of the item
      // before is issued (it reads the dS columns they overwrite)
      while (ok && cur.u < n_units) {
        Cur nx = cur;
        advance(nx);
        if (nx.u < n_units && !(ok = issue_sp(nx, jj + 1))) break;
        const int s = jj & 1, sk = jj % NKS;
        if (!(ok = mbar_wait(&bars[DP_DS + s], (jj >> 1) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint64_t dkm = desc_add(dkm0, sk * L::KV);
        const uint32_t tA = tmem + 128 + s * BNK;
#pragma unroll
        for (int kk = 0; kk < BNK / 16; ++kk) {
          // keys 16kk..16kk+15: packed in the half (kk/2) written by warp group kk/2
          const uint32_t acol = (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8);
          mma_bf16_ts(tDQ, tA + acol, desc_add(dkm, kk * 2048), idDQ, (cur.j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars[DP_KVE + sk]);
        if (cur.j == cur.t.nk - 1) mma_commit(&bars[DP_ACC]);
        cur = nx;
        ++jj;
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    // warps 2..9: row = TMEM lane = query; warps w and w+4 share a lane
    // quarter and split the columns (half 0 / half 1), two warps per scheduler
    const int half = (warp - 2) >> 2;
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const float sc = g.scale * kLog2e;
    // this row's lse*log2(e) / D, loaded one unit ahead
    auto fetch = [&](int u, float& l2, float& dd) {
      l2 = INFINITY;
      dd = 0.f;
      if (u < n_units) {
        const DqUnit t = dq_unit<BNK>(g, u);
        const int tq = t.q0 + row;
        if (tq < g.T) {
          l2 = __ldg(lse + ((int64_t)t.b * g.H + t.h) * g.T + tq) * kLog2e;
          dd = __ldg(delta + ((int64_t)t.b * g.H + t.h) * g.T + tq);
        }
      }
    };
    float nlse2, ndt;
    fetch(blockIdx.x, nlse2, ndt);
    int jj = 0, n = 0, m = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++n) {
      const DqUnit t = dq_unit<BNK>(g, u);
      const int qb = n & 1;
      const float lse2 = nlse2, dt = ndt;
      fetch(u + gridDim.x, nlse2, ndt);
      const int tq = t.q0 + row;
      const int lo = tq < g.T ? local_lo(g, tq) : 0x7fffffff;
      for (int j = 0; j < t.nk; ++j, ++jj) {
        const int s = jj & 1;
        // S(jj) done implies the dQ MMA of item jj-2 (issued earlier) has
        // finished reading the dS columns this pass overwrites
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[DP_SP + s], (jj >> 1) & 1, abort, &g_fault_word));
        if (!ok) break;
        tc_fence_after();
        const int k0 = t.kbase + j * BNK;
        const int c_lo = lo - k0, c_hi = tq - k0;
        const int cc = half;  // this warp's 32 of the tile's 64 key columns
        uint32_t rs[32], rp[32];
        tmem_ld32(tmem + lane_off + s * BNK + cc * 32, rs);
        tmem_ld32(tmem + lane_off + 128 + s * BNK + cc * 32, rp);
        tmem_ld_wait();
        uint32_t pk[16];
        // interior tiles (all 32 keys visible from every query of the warp) skip the mask
        const bool full = __all_sync(0xffffffffu, c_lo <= cc * 32 && c_hi >= cc * 32 + 32);
        const uint64_t sc2 = f2_pack(sc, sc), nl2 = f2_pack(-lse2, -lse2), dt2 = f2_pack(dt, dt);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = cc * 32 + 2 * i;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(rs[2 * i]), __uint_as_float(rs[2 * i + 1])), sc2, nl2), x0, x1);
          float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          if (!full) {
            p0 = (c >= c_lo && c < c_hi) ? p0 : 0.f;
            p1 = (c + 1 >= c_lo && c + 1 < c_hi) ? p1 : 0.f;
          }
          float d0, d1;
          f2_unpack(f2_mul(f2_pack(p0, p1),
                           f2_sub(f2_pack(__uint_as_float(rp[2 * i]), __uint_as_float(rp[2 * i + 1])), dt2)),
                    d0, d1);
          pk[i] = pack_bf16(d0, d1);
        }
        tmem_st16(tmem + lane_off + 128 + s * BNK + cc * 32, pk);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars[DP_DS + s]);
      }
      if (!ok) break;
      // epilogue: dQ (scaled) as bf16 128-byte-swizzled 64-column panels over
      // the unit's Q tile (free once the unit's MMAs are done), then TMA
      // stores (rows >= T clipped by the map)
      if (t.nk > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[DP_ACC], m & 1, abort, &g_fault_word));
      else  // no MMAs: only make sure the unit's Q copy has landed before overwriting it
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[DP_Q + qb], (n >> 1) & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      uint8_t* stage = smem + qb * L::QD + L::Q;
#pragma unroll
      for (int cc = half * (HD / 64); cc < (half + 1) * (HD / 64); ++cc) {
        uint32_t r[32];
        if (t.nk > 0) {
          tmem_ld32(tDQ + lane_off + cc * 32, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16(__uint_as_float(r[2 * i]) * g.scale, __uint_as_float(r[2 * i + 1]) * g.scale);
        uint8_t* prow = stage + (cc >> 1) * (BM * 128) + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = (cc & 1) * 4 + q;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (row & 7)) * 16)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      if (t.nk > 0) {
        tc_fence_before();
        ++m;
      }
      fence_async_smem();
      mbar_arrive(&bars[DP_STG]);
      if (warp == 2 && lane == 0) {
        // all 256 staging writes done -> store dQ; buffer qb free once read
        ok = mbar_wait(&bars[DP_STG], n & 1, abort, &g_fault_word);
        if (ok) {
#pragma unroll
          for (int p = 0; p < HD / 64; ++p) tma_store_4d(&tm_st, stage + p * (BM * 128), p * 64, t.h, t.q0, t.b);
          tma_store_commit();
          tma_store_wait_read();
          mbar_arrive(&bars[DP_QE + qb]);
        }
      }
      ok = __all_sync(0xffffffffu, ok);
    }
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// dk, dv: persistent. Each CTA walks work units u = blockIdx.x + k * gridDim.x
// (unit = 128 keys of one (b, h), heads fastest). The Q/dO ring and the
// S^T/dP^T buffers run on counters that continue across units, so the next
// unit's first query tiles load while the current one finishes; its K/V load
// once the current unit's dK/dV, staged in the K/V region, have been stored.
// Launch-aligned waves of non-persistent CTAs all load at once and all store
// at once; a persistent walk spreads both over time.

template <int HD>
struct DkvLayout {
  static constexpr int BNQ = 64;                   // queries per inner tile
  static constexpr int NQS = 3;                    // Q / dO stages
  static constexpr int KPANEL = BM * 128;          // 128-key panel (16 KB)
  static constexpr int QPANEL = BNQ * 128;         // 64-query panel (8 KB)
  static constexpr int KTILE = BM * HD * 2;
  static constexpr int QTILE = BNQ * HD * 2;
  // two K/V buffers: unit n uses buffer n&1, so the next unit's K/V load
  // while this one finishes (its dK/dV are staged over its own K/V tiles)
  static constexpr int KV = 2 * KTILE;             // bytes of one K/V buffer
  static constexpr int K = 0;                      // + kb * KV: K tile, then dK staging
  static constexpr int V = K + KTILE;              // + kb * KV: V tile, then dV staging
  static constexpr int Q = 2 * KV;                 // NQS stages
  static constexpr int DO = Q + NQS * QTILE;       // NQS stages
  static constexpr int VEC = DO + NQS * QTILE;     // per compute warp: {-lse*log2e, D}[32]
  static constexpr int BAR = VEC + 8 * 2 * 32 * 4;
  static constexpr int BYTES = BAR + 256;
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

// barriers: K/V loaded / K,V region free again (dK, dV stores have read it);
// per Q/dO stage loaded / released; per TMEM buffer S^T,dP^T ready /
// P^T,dS^T written; dV,dK complete / read out of TMEM; dK,dV staged
enum {
  KV_KV = 0, KV_KVE = 2, KV_QD = 4, KV_QDE = 8, KV_SP = 12, KV_PD = 14, KV_ACC = 16, KV_ACCE = 17, KV_STG = 18,
  KV_NB = 19
};

struct DkvUnit {
  int h, k0, b, tfirst, tlast, nq;
};
__device__ __forceinline__ DkvUnit dkv_unit(const Geom& g, int u) {
  DkvUnit t;
  const int nkt = cdiv(g.T, BM);
  t.h = u % g.H;
  const int r = u / g.H;
  t.k0 = (r % nkt) * BM;
  t.b = r / nkt;
  t.tfirst = t.k0 + 1;
  t.tlast = min(g.T - 1, t.k0 + BM - 1 + g.W);
  t.nq = t.tlast >= t.tfirst ? (t.tlast - t.tfirst + 64) / 64 : 0;
  return t;
}

template <int HD>
__global__ void __launch_bounds__(320, 1)
    local_dkv_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv128, const __grid_constant__ CUtensorMap tm_qkv64,
                        const __grid_constant__ CUtensorMap tm_do64, const __grid_constant__ CUtensorMap tm_st,
                        Geom g, const float* __restrict__ lse, const float* __restrict__ delta, int n_units) {
  using L = DkvLayout<HD>;
  constexpr int BNQ = L::BNQ, NQS = L::NQS;
  extern __shared__ __align__(1024) uint8_t smem_dkv[];
  uint8_t* smem = smem_dkv;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + KV_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {  // the swizzled layouts need 1024-byte alignment
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int kb = 0; kb < 2; ++kb) {
      mbar_init(&bars[KV_KV + kb], 1);
      mbar_init(&bars[KV_KVE + kb], 1);
    }
    for (int s = 0; s < NQS; ++s) {
      mbar_init(&bars[KV_QD + s], 1);
      mbar_init(&bars[KV_QDE + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[KV_SP + s], 1);
      mbar_init(&bars[KV_PD + s], 2 * BM);
    }
    mbar_init(&bars[KV_ACC], 1);
    mbar_init(&bars[KV_ACCE], 2 * BM);
    mbar_init(&bars[KV_STG], 2 * BM);
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
  // S^T at [0,64) / [64,128), dP^T at [128,192) / [192,256), dV, dK after.
  // P^T and dS^T (bf16) are written back over the first 16 of each 32
  // S^T / dP^T columns that produced them and feed the dV / dK MMAs from TMEM.
  const uint32_t tDV = tmem + 256, tDK = tmem + 256 + HD;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_qkv128);
      prefetch_tmap(&tm_qkv64);
      prefetch_tmap(&tm_do64);
      prefetch_tmap(&tm_st);
      int q = 0, n = 0, issued_q = 0, issued_kv = 0;
      bool ok = true;
      auto load_qd = [&](const DkvUnit& t, int i) -> bool {
        const int gq = q + i, s = gq % NQS;
        if (gq >= NQS && !mbar_wait(&bars[KV_QDE + s], ((gq / NQS) - 1) & 1, abort, &g_fault_word)) return false;
        const int t0 = t.tfirst + i * BNQ;
        mbar_expect_tx(&bars[KV_QD + s], 2 * L::QTILE);
        tma_load_tile<HD / 64, 64>(&tm_qkv64, &bars[KV_QD + s], smem + L::Q + s * L::QTILE, t0, t.h, t.b);
        tma_load_tile<HD / 64, 64>(&tm_do64, &bars[KV_QD + s], smem + L::DO + s * L::QTILE, t0, t.h, t.b);
        issued_q = gq + 1;
        return true;
      };
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++n) {
        const DkvUnit t = dkv_unit(g, u);
        // K/V buffer n&1: free once unit n-2's dK/dV stores have read it
        const int kb = n & 1;
        if (n >= 2 && !(ok = mbar_wait(&bars[KV_KVE + kb], ((n >> 1) - 1) & 1, abort, &g_fault_word))) break;
        mbar_expect_tx(&bars[KV_KV + kb], 2 * L::KTILE);
        tma_load_tile<HD / 64, BM>(&tm_qkv128, &bars[KV_KV + kb], smem + kb * L::KV + L::K, t.k0, g.H + t.h, t.b);
        tma_load_tile<HD / 64, BM>(&tm_qkv128, &bars[KV_KV + kb], smem + kb * L::KV + L::V, t.k0, 2 * g.H + t.h, t.b);
        issued_kv = n + 1;
        for (int i = 0; ok && i < t.nq; ++i) ok = load_qd(t, i);
        q += t.nq;
      }
      if (!ok) {
        raise_fault(g, kFaultProducer, abort);
        // let the copies already issued land before the CTA can exit
        volatile int none = 0;
        volatile unsigned gnone = 0;
        if (issued_kv > 0)
          mbar_wait(&bars[KV_KV + ((issued_kv - 1) & 1)], ((issued_kv - 1) >> 1) & 1, &none, &gnone, 100000000ull);
        for (int gq = issued_q - NQS < 0 ? 0 : issued_q - NQS; gq < issued_q; ++gq)
          mbar_wait(&bars[KV_QD + gq % NQS], (gq / NQS) & 1, &none, &gnone, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idSP = idesc_bf16_f32(BM, BNQ, false, false);  // K Q^T, V dO^T
      constexpr uint32_t idKV = idesc_bf16_f32(BM, HD, false, true);    // P^T dO, dS^T Q
      const uint64_t dkb0 = desc_sw128(smem_u32(smem + L::K), 16, 1024);
      const uint64_t dvb0 = desc_sw128(smem_u32(smem + L::V), 16, 1024);
      int q = 0, n = 0, m = 0;  // m: units with at least one query tile
      bool ok = true;
      auto issue_sp = [&](int gq, uint64_t dk0, uint64_t dv0) -> bool {
        const int s = gq & 1, sq = gq % NQS;
        if (!mbar_wait(&bars[KV_QD + sq], (gq / NQS) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint64_t dq = desc_sw128(smem_u32(smem + L::Q + sq * L::QTILE), 16, 1024);
        const uint64_t ddo = desc_sw128(smem_u32(smem + L::DO + sq * L::QTILE), 16, 1024);
        const uint32_t tS = tmem + s * BNQ, tP = tmem + 128 + s * BNQ;
        // K steps past a padded head_dim would multiply zero-filled columns: skipped
#pragma unroll
        for (int kk = 0; kk < HD / 16 && kk * 16 < g.hd; ++kk) {
          const uint32_t aoff = (kk / 4) * L::KPANEL + (kk % 4) * 32;
          const uint32_t boff = (kk / 4) * L::QPANEL + (kk % 4) * 32;
          mma_bf16(tS, desc_add(dk0, aoff), desc_add(dq, boff), idSP, kk > 0);
          mma_bf16(tP, desc_add(dv0, aoff), desc_add(ddo, boff), idSP, kk > 0);
        }
        mma_commit(&bars[KV_SP + s]);
        return true;
      };
      // S^T(i+1) is issued before dV/dK(i): the softmax warps wait for it
      // next, and it may start once dV/dK(i-1) are issued (they read the
      // P^T columns S^T(i+1) overwrites)
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++n) {
        const DkvUnit t = dkv_unit(g, u);
        const int kb = n & 1;
        if (!(ok = mbar_wait(&bars[KV_KV + kb], (n >> 1) & 1, abort, &g_fault_word))) break;
        const uint64_t dk0 = desc_add(dkb0, kb * L::KV), dv0 = desc_add(dvb0, kb * L::KV);
        tc_fence_after();
        if (t.nq > 0) {
          ok = issue_sp(q, dk0, dv0);
          for (int i = 0; ok && i < t.nq; ++i) {
            const int gq = q + i, s = gq & 1, sq = gq % NQS;
            if (i + 1 < t.nq && !(ok = issue_sp(gq + 1, dk0, dv0))) break;
            if (!(ok = mbar_wait(&bars[KV_PD + s], (gq >> 1) & 1, abort, &g_fault_word))) break;
            // the first dV/dK MMA overwrites the accumulators: the previous
            // unit's epilogue must have read them
            if (i == 0 && m > 0 && !(ok = mbar_wait(&bars[KV_ACCE], (m - 1) & 1, abort, &g_fault_word))) break;
            tc_fence_after();
            const uint64_t dqm = desc_sw128(smem_u32(smem + L::Q + sq * L::QTILE), L::QPANEL, 1024);
            const uint64_t ddom = desc_sw128(smem_u32(smem + L::DO + sq * L::QTILE), L::QPANEL, 1024);
            const uint32_t tA = tmem + s * BNQ;
#pragma unroll
            for (int kk = 0; kk < BNQ / 16; ++kk) {
              const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
              // queries 16kk..16kk+15: packed in the half (kk/2) written by warp group kk/2
              const uint32_t acol = (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8);
              mma_bf16_ts(tDV, tA + acol, desc_add(ddom, kk * 2048), idKV, acc);
              mma_bf16_ts(tDK, tA + 128 + acol, desc_add(dqm, kk * 2048), idKV, acc);
            }
            mma_commit(&bars[KV_QDE + sq]);
          }
          if (!ok) break;
          mma_commit(&bars[KV_ACC]);
          ++m;
        }
        q += t.nq;
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    // warps 2..9: row = TMEM lane = key; warps w and w+4 split the columns
    const int half = (warp - 2) >> 2;
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const float sc = g.scale * kLog2e;
    float* v_lse = reinterpret_cast<float*>(smem + L::VEC) + (warp - 2) * 64;
    float* v_d = v_lse + 32;
    int q = 0, n = 0, m = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++n) {
      const DkvUnit t = dkv_unit(g, u);
      const int j = t.k0 + row;  // this thread's key
      const bool valid = j < g.T;
      // queries that see key j form one range: t in (j, j+W] with qs(t) <= j+W-1,
      // i.e. t < the end of the bsL-block holding j+W-1 (mask of models.py:286-292)
      const int t_hi = local_hi(g, j);  // inclusive
      const float* lse_b = lse + ((int64_t)t.b * g.H + t.h) * g.T;
      const float* d_b = delta + ((int64_t)t.b * g.H + t.h) * g.T;
      // this lane's -lse*log2(e) / D for the next query tile, loaded one tile ahead
      auto fetch = [&](int i, float& l2, float& dd) {
        const int tq = t.tfirst + i * BNQ + half * 32 + lane;
        const bool tv = i < t.nq && tq <= t.tlast;
        l2 = tv ? -__ldg(lse_b + tq) * kLog2e : -INFINITY;
        dd = tv ? __ldg(d_b + tq) : 0.f;
      };
      float nl2, nd;
      fetch(0, nl2, nd);
      for (int i = 0; i < t.nq; ++i) {
        const int gq = q + i, s = gq & 1;
        const int t0 = t.tfirst + i * BNQ;
        __syncwarp();
        v_lse[lane] = nl2;
        v_d[lane] = nd;
        __syncwarp();
        fetch(i + 1, nl2, nd);
        // S^T(gq) done implies the dV/dK MMAs of tile gq-2 (issued earlier)
        // have finished reading the P^T / dS^T columns this pass overwrites
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[KV_SP + s], (gq >> 1) & 1, abort, &g_fault_word));
        if (!ok) break;
        tc_fence_after();
        const int c_lo = j + 1 - t0 - half * 32, c_hi = valid ? t_hi - t0 - half * 32 + 1 : -1;  // in [0, 32)
        {
          const int cc = half;
          uint32_t rs[32], rp[32];
          tmem_ld32(tmem + lane_off + s * BNQ + cc * 32, rs);
          tmem_ld32(tmem + lane_off + 128 + s * BNQ + cc * 32, rp);
          tmem_ld_wait();
          uint32_t pp[16], pd[16];
          // interior tiles (every key of the warp sees all 32 queries) skip the mask
          const bool full = __all_sync(0xffffffffu, c_lo <= 0 && c_hi >= 32);
          const float4* nl4 = reinterpret_cast<const float4*>(v_lse);
          const float4* d4 = reinterpret_cast<const float4*>(v_d);
          const uint64_t sc2 = f2_pack(sc, sc);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 nl = nl4[q4], dd = d4[q4];
#pragma unroll
            for (int uu = 0; uu < 2; ++uu) {
              const int c = 4 * q4 + 2 * uu;
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sc2,
                               uu == 0 ? f2_pack(nl.x, nl.y) : f2_pack(nl.z, nl.w)),
                        x0, x1);
              float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
              if (!full) {
                p0 = (c >= c_lo && c < c_hi) ? p0 : 0.f;
                p1 = (c + 1 >= c_lo && c + 1 < c_hi) ? p1 : 0.f;
              }
              const uint64_t ds = f2_mul(f2_pack(p0, p1),
                                         f2_sub(f2_pack(__uint_as_float(rp[c]), __uint_as_float(rp[c + 1])),
                                                uu == 0 ? f2_pack(dd.x, dd.y) : f2_pack(dd.z, dd.w)));
              float d0, d1;
              f2_unpack(ds, d0, d1);
              pp[c / 2] = pack_bf16(p0, p1);
              pd[c / 2] = pack_bf16(d0, d1);
            }
          }
          tmem_st16(tmem + lane_off + s * BNQ + cc * 32, pp);
          tmem_st16(tmem + lane_off + 128 + s * BNQ + cc * 32, pd);
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(&bars[KV_PD + s]);
      }
      if (!ok) break;
      // epilogue: dK (half 0, scaled) / dV (half 1) as bf16 128-byte-swizzled
      // 64-column panels over the K / V tiles (free once the unit's MMAs are
      // done), then TMA stores (rows >= T clipped by the map)
      if (t.nq > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[KV_ACC], m & 1, abort, &g_fault_word));
      else  // no MMAs: only make sure the unit's K/V copy has landed before overwriting it
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[KV_KV + (n & 1)], (n >> 1) & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      uint8_t* stage = smem + (n & 1) * L::KV + (half == 0 ? L::K : L::V);
      const uint32_t tsrc = (half == 0 ? tDK : tDV) + lane_off;
      const float mul = half == 0 ? g.scale : 1.f;
#pragma unroll
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t r[32];
        if (t.nq > 0) {
          tmem_ld32(tsrc + cc * 32, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i2 = 0; i2 < 32; ++i2) r[i2] = 0u;
        }
        uint32_t pk[16];
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2)
          pk[i2] = pack_bf16(__uint_as_float(r[2 * i2]) * mul, __uint_as_float(r[2 * i2 + 1]) * mul);
        uint8_t* prow = stage + (cc >> 1) * (BM * 128) + row * 128;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int chunk = (cc & 1) * 4 + qq;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (row & 7)) * 16)) =
              make_uint4(pk[4 * qq], pk[4 * qq + 1], pk[4 * qq + 2], pk[4 * qq + 3]);
        }
      }
      if (t.nq > 0) {
        tc_fence_before();
        mbar_arrive(&bars[KV_ACCE]);
        ++m;
      }
      fence_async_smem();
      mbar_arrive(&bars[KV_STG]);
      if (warp == 2 && lane == 0) {
        // all 256 staging writes done -> store dK, dV; K/V region free once read
        ok = mbar_wait(&bars[KV_STG], n & 1, abort, &g_fault_word);
        if (ok) {
#pragma unroll
          for (int p = 0; p < HD / 64; ++p) {
            tma_store_4d(&tm_st, smem + (n & 1) * L::KV + L::K + p * (BM * 128), p * 64, g.H + t.h, t.k0, t.b);
            tma_store_4d(&tm_st, smem + (n & 1) * L::KV + L::V + p * (BM * 128), p * 64, 2 * g.H + t.h, t.k0, t.b);
          }
          tma_store_commit();
          tma_store_wait_read();
          mbar_arrive(&bars[KV_KVE + (n & 1)]);
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      q += t.nq;
    }
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
