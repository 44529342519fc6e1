// Forward of the tensor-core local branch, sized for two CTAs per SM
// (included by local_sm100.cu).
//
// One CTA per (batch, head, 128-query tile); 6 warps:
//   warp 0     TMA producer: Q tile, then 64-key K/V tiles into a 2-stage ring
//   warp 1     TMEM allocator (256 columns) and single-thread MMA issuer:
//              S_j = Q K_j^T (M128 N64) into one of two TMEM buffers,
//              O += P_j V_j (M128 N=hd), and at the end the fused remote tile
//              R = lat W_h^T into the freed S columns
//   warps 2-5  softmax: thread r owns query row r (TMEM lane r); online
//              softmax with the window mask, P_j bf16 into swizzled smem, O
//              rescaled in TMEM when the running max moves; epilogue writes
//              local_out, lse and (fused) the gated mix with the remote row.
// 256 TMEM columns and <= 113 KB of shared memory per CTA let two CTAs share
// an SM, so one CTA's load / epilogue latency hides behind the other's work.

template <int HD>
struct Fwd2Layout {
  static constexpr int BNK = 64;
  static constexpr int QPANEL = BM * 128;    // 128 rows x 128 bytes
  static constexpr int KPANEL = BNK * 128;   // 64 rows x 128 bytes
  static constexpr int QTILE = BM * HD * 2;
  static constexpr int KTILE = BNK * HD * 2;
  static constexpr int Q = 0;
  static constexpr int K = Q + QTILE;        // 2 stages
  static constexpr int V = K + 2 * KTILE;    // 2 stages
  static constexpr int P = V + 2 * KTILE;    // 128 x 64 bf16
  // the fused gate's lat tile and W_rout slice reuse the K stages after the
  // last S MMA has completed
  static constexpr int LAT = K;
  static constexpr int WR = K + BM * 128;
  static constexpr int BAR = P + BM * BNK * 2;
  static constexpr int BYTES = BAR + 128;
};

enum { F_Q = 0, F_K = 1, F_V = 3, F_KVE = 5, F_S = 7, F_P = 9, F_O = 10, F_LW = 11, F_R = 12, F_NB = 13 };

template <int HD>
__global__ void __launch_bounds__(192, 2)
    local_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv, Geom g,
                        bf16* __restrict__ local_out, float* __restrict__ lse_out, GateEpilogue ep) {
  using L = Fwd2Layout<HD>;
  constexpr int BNK = L::BNK;
  extern __shared__ __align__(1024) uint8_t smem_fwd[];
  uint8_t* smem = smem_fwd;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + F_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // the 128-byte swizzle needs 1024-byte aligned tiles; the launch requests
  // no slack, so a misaligned window is reported instead of computed on
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicOr(&g_fault_word, kFaultEpilogue);
    return;
  }

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = blockIdx.x * BM;
  const int qlast = min(q0 + BM - 1, g.T - 1);
  const int kbase = local_lo(g, q0);
  const int khi = qlast - 1;
  const int nk = khi >= kbase ? (khi - kbase + BNK) / BNK : 0;
  const bool fuse = ep.lat != nullptr;

  if (threadIdx.x == 0) {
    mbar_init(&bars[F_Q], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[F_K + s], 1);
      mbar_init(&bars[F_V + s], 1);
      mbar_init(&bars[F_KVE + s], 1);
      mbar_init(&bars[F_S + s], 1);
    }
    mbar_init(&bars[F_P], BM);
    mbar_init(&bars[F_O], 1);
    mbar_init(&bars[F_LW], BM);
    mbar_init(&bars[F_R], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 128, tR = tmem;  // S buffers at [0,64) and [64,128); R reuses them

  if (warp == 0) {
    if (lane == 0 && nk > 0) {
      int issued = 0;
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_kv);
      mbar_expect_tx(&bars[F_Q], L::QTILE);
#pragma unroll
      for (int p = 0; p < HD / 64; ++p) tma_load_4d(&tm_q, &bars[F_Q], smem + L::Q + p * L::QPANEL, p * 64, h, q0, b);
      for (int j = 0; j < nk; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bars[F_KVE + s], ((j >> 1) - 1) & 1, abort, &g_fault_word)) {
          raise_fault(kFaultProducer, abort);
          break;
        }
        const int k0 = kbase + j * BNK;
        mbar_expect_tx(&bars[F_K + s], L::KTILE);
#pragma unroll
        for (int p = 0; p < HD / 64; ++p)
          tma_load_4d(&tm_kv, &bars[F_K + s], smem + L::K + s * L::KTILE + p * L::KPANEL, p * 64, g.H + h, k0, b);
        mbar_expect_tx(&bars[F_V + s], L::KTILE);
#pragma unroll
        for (int p = 0; p < HD / 64; ++p)
          tma_load_4d(&tm_kv, &bars[F_V + s], smem + L::V + s * L::KTILE + p * L::KPANEL, p * 64, 2 * g.H + h, k0,
                      b);
        issued = j + 1;
      }
      if (*abort) {
        volatile int none = 0;
        volatile unsigned gnone = 0;
        mbar_wait(&bars[F_Q], 0, &none, &gnone, 100000000ull);
        for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
          mbar_wait(&bars[F_K + (j & 1)], (j >> 1) & 1, &none, &gnone, 100000000ull);
          mbar_wait(&bars[F_V + (j & 1)], (j >> 1) & 1, &none, &gnone, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && (nk > 0 || fuse)) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BNK, false, false);
      constexpr uint32_t idO = idesc_bf16_f32(BM, HD, false, true);
      const uint32_t q_addr = smem_u32(smem + L::Q);
      const uint32_t p_addr = smem_u32(smem + L::P);
      bool ok = true;
      if (nk > 0) ok = mbar_wait(&bars[F_Q], 0, abort, &g_fault_word);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&bars[F_K + s], (j >> 1) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::K + s * L::KTILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_bf16(tmem + s * BNK, desc_sw128(q_addr + (kk / 4) * L::QPANEL + (kk % 4) * 32, 16, 1024),
                   desc_sw128(k_addr + (kk / 4) * L::KPANEL + (kk % 4) * 32, 16, 1024), idS, kk > 0);
        mma_commit(&bars[F_S + s]);
        return true;
      };
      if (ok && nk > 0) ok = issue_s(0);
      for (int j = 0; ok && j < nk; ++j) {
        if (j + 1 < nk && !(ok = issue_s(j + 1))) break;
        if (!(ok = mbar_wait(&bars[F_P], j & 1, abort, &g_fault_word))) break;
        if (!(ok = mbar_wait(&bars[F_V + (j & 1)], (j >> 1) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + L::V + (j & 1) * L::KTILE);
#pragma unroll
        for (int kk = 0; kk < BNK / 16; ++kk)
          mma_bf16(tO, desc_sw128(p_addr + kk * 32, 16, 1024), desc_sw128(v_addr + kk * 2048, L::KPANEL, 1024), idO,
                   (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars[F_KVE + (j & 1)]);
        mma_commit(&bars[F_O]);
      }
      if (ok && fuse) {
        // remote tile R = lat_tile (128 x 64) . W_h^T (64 x hd), written by the
        // softmax warps into the K stages once every S MMA had completed
        ok = mbar_wait(&bars[F_LW], 0, abort, &g_fault_word);
        if (ok) {
          tc_fence_after();
          constexpr uint32_t idR = idesc_bf16_f32(BM, HD, false, false);
          const uint32_t la = smem_u32(smem + L::LAT), wa = smem_u32(smem + L::WR);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tR, desc_sw128(la + kk * 32, 16, 1024), desc_sw128(wa + kk * 32, 16, 1024), idR, kk > 0);
          mma_commit(&bars[F_R]);
        }
      }
      if (!ok) raise_fault(kFaultMma, abort);
    }
  } else {
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const int t = q0 + row;
    const bool valid = t < g.T;
    const int lo = valid ? local_lo(g, t) : 0x7fffffff;
    const float sc = g.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    uint8_t* prow = smem + L::P + row * 128;
    bool ok = true;
    for (int j = 0; ok && j < nk; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[F_S + s], (j >> 1) & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tsrc = tmem + s * BNK + lane_off;
      const int c_lo = lo - (kbase + j * BNK);  // visible columns: [c_lo, c_hi)
      const int c_hi = t - (kbase + j * BNK);
      uint32_t r0[32], r1[32];
      tmem_ld32(tsrc, r0);
      tmem_ld32(tsrc + 32, r1);
      tmem_ld_wait();
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (i >= c_lo && i < c_hi) mx = fmaxf(mx, __uint_as_float(r0[i]));
        if (i + 32 >= c_lo && i + 32 < c_hi) mx = fmaxf(mx, __uint_as_float(r1[i]));
      }
      const float m_new = fmaxf(m, mx * sc);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);
      // P buffer and O are free once PV_{j-1} has completed
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[F_O], (j - 1) & 1, abort, &g_fault_word));
        if (!ok) break;
      }
      tc_fence_after();
      float psum = 0.f;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = cc * 32 + 2 * i;
          const float s0 = __uint_as_float(cc ? r1[2 * i] : r0[2 * i]);
          const float s1 = __uint_as_float(cc ? r1[2 * i + 1] : r0[2 * i + 1]);
          const float p0 = (c >= c_lo && c < c_hi) ? exp2f(s0 * sc - m_use) : 0.f;
          const float p1 = (c + 1 >= c_lo && c + 1 < c_hi) ? exp2f(s1 * sc - m_use) : 0.f;
          psum += p0 + p1;
          pk[i] = pack_bf16(p0, p1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = cc * 4 + q;
          *reinterpret_cast<uint4*>(prow + (((chunk & 7) ^ (row & 7)) * 16)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      fence_async_smem();
      l = l * alpha + psum;
      m = m_new;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int cc = 0; cc < HD / 32; ++cc) {
          uint32_t r[32];
          tmem_ld32(tO + lane_off + cc * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(tO + lane_off + cc * 32, r);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(&bars[F_P]);
    }
    if (!ok) raise_fault(kFaultSoftmax, abort);
    if (ok && nk > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars[F_O], (nk - 1) & 1, abort, &g_fault_word));
    if (ok && fuse) {
      // every MMA has completed: the K stages hold the lat tile and W_h now
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const bf16*>(ep.lat) +
                                                        ((int64_t)b * g.Tq + (valid ? t / g.qbs : 0)) * 64);
      uint8_t* dl_ = smem + L::LAT + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dl_ + ((c ^ (row & 7)) * 16)) = src[c];
      if (row < HD) {
        const uint4* wsrc =
            reinterpret_cast<const uint4*>(static_cast<const bf16*>(ep.w_rout) + ((int64_t)h * HD + row) * 64);
        uint8_t* wd = smem + L::WR + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(wd + ((c ^ (row & 7)) * 16)) = wsrc[c];
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[F_LW]);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[F_R], 0, abort, &g_fault_word));
    }
    if (!ok) {
      raise_fault(kFaultEpilogue, abort);
    } else {
      // epilogue; TMEM loads are warp-collective, rows past T skip the stores
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* dst = local_out + ((int64_t)b * g.T + (valid ? t : 0)) * g.d + (int64_t)h * HD;
      if (fuse) {
        const float4* bh4 = reinterpret_cast<const float4*>(ep.b_rout + (int64_t)h * HD);
        const float4* gl4 = reinterpret_cast<const float4*>(ep.g_local);
        const float4* gr4 = reinterpret_cast<const float4*>(ep.g_remote);
        // pass A: gate logits from the bf16-rounded local row (the value stored
        // for the backward) and the remote row
        float sl = 0.f, sr = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < HD / 32; ++cc) {
          uint32_t ro[32], rr[32];
          if (nk > 0) tmem_ld32(tO + lane_off + cc * 32, ro);
          tmem_ld32(tR + lane_off + cc * 32, rr);
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
        const float x = sl + g.gate_bias - sr;
        const float wl = 1.f / (1.f + expf(-x));
        const float wr = 1.f / (1.f + expf(x));
        bf16* mdst = static_cast<bf16*>(ep.mixed) + ((int64_t)b * g.T + (valid ? t : 0)) * g.d + (int64_t)h * HD;
#pragma unroll 1
        for (int cc = 0; cc < HD / 32; ++cc) {
          uint32_t ro[32], rr[32];
          if (nk > 0) tmem_ld32(tO + lane_off + cc * 32, ro);
          tmem_ld32(tR + lane_off + cc * 32, rr);
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
      } else {
#pragma unroll 1
        for (int cc = 0; cc < HD / 32; ++cc) {
          uint32_t r[32];
          if (nk > 0) {
            tmem_ld32(tO + lane_off + cc * 32, r);
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
      if (valid) lse_out[((int64_t)b * g.H + h) * g.T + t] = l > 0.f ? (m + log2f(l)) * kLn2 : INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}
