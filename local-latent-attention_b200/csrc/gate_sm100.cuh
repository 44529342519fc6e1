// Gate / r_out backward on the tensor cores (included by local_sm100.cu).
//
// gate_bwd: one CTA per (b, 128-token tile), looping over the H heads. Per
// head h, with remote R_h = lat[t/qbs] W_h^T + b_h recomputed by one MMA:
//   x = L.g_l + bias - R.g_r, w = sigmoid(x), ds = (dm.(L - R)) w (1 - w)
//   dL = w dm + ds g_l  (bf16, read by the local backward), D = dL.L
//   dR = (1 - w) dm - ds g_r  (bf16, read by the dW GEMM)
//   dlat += dR_h W_h    (MMA, accumulated over heads in TMEM)
//   dg_l += ds L, dg_r -= ds R  (warp butterfly reductions, per-CTA partial)
// Warps: 1 = TMEM + MMA issuer, 2-5 = one token row per thread, 0 idle.
//
// rout_dw: dW_rout[c, e] = sum_t dR[t, c] lat[t/qbs, e], db[c] = sum_t dR[t, c];
// one CTA per (128 columns of d, token split), 64-token K steps, dR tiles by
// TMA (MN-major A operand), lat tiles written by threads (MN-major B), the
// column sums for db taken from the same shared-memory tiles.

// G warp groups per CTA, each taking every G-th head with its own buffers.
// G = 2: 512 TMEM columns, ~200 KB of shared memory, one CTA per SM.
// G = 1: 256 TMEM columns and < 113 KB, two CTAs per SM: one CTA's head chain
// (load, two passes, stores) overlaps the other's.
template <int G>
constexpr int gate_max_heads() { return G == 2 ? 32 : 24; }  // per-head ds rows kept in shared memory
constexpr int kGateMaxHeads = 32;

// floats per CTA in dg_part: dg_local [hd], then S1_h [64] and S0_h per head
__host__ __device__ constexpr int gate_dg_stride(int hd, int H) { return hd + H * 65; }

// dg_remote[c] = -sum_h (sum_e S1_h[e] W[h*hd + c, e] + S0_h b[h*hd + c])
// from the reduced gate partials (dg_sum + hd). Block = 16 columns; its 256
// threads = 16 columns x 16 slices of the (head, 8-wide e chunk) pairs,
// summed over the slices in a fixed order.
__global__ void __launch_bounds__(256) gate_dgr_finalize_kernel(Geom g, const float* __restrict__ dg_sum,
                                                                const bf16* __restrict__ w_rout,
                                                                const float* __restrict__ b_rout,
                                                                float* __restrict__ dg_remote) {
  __shared__ float part[16][17];
  const int HD = g.hd, H = g.H;
  const float* s1 = dg_sum + HD;
  const int cl = threadIdx.x & 15, sl = threadIdx.x >> 4;
  const int c = blockIdx.x * 16 + cl;
  float v = 0.f;
  if (c < HD) {
    for (int it = sl; it < H * 9; it += 16) {  // per head: 8 chunks of W_h[c, :] and the bias term
      const int h = it / 9, q = it % 9;
      const float* sh = s1 + h * 65;
      if (q < 8) {
        float wv[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(w_rout + ((int64_t)h * HD + c) * 64) + q), wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) v = fmaf(sh[q * 8 + k], wv[k], v);
      } else {
        v = fmaf(sh[64], b_rout[(int64_t)h * HD + c], v);
      }
    }
  }
  part[sl][cl] = v;
  __syncthreads();
  if (sl == 0 && c < HD) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) t += part[k][cl];
    dg_remote[c] = -t;
  }
}

template <int HD, int G = 2>
struct GbLayout {
  static constexpr int TILE = BM * HD * 2;         // 128 rows x HD bf16 (HD/64 panels of 16 KB)
  static constexpr int LAT = 0;                    // 128 x 64 bf16
  static constexpr int W = LAT + BM * 128;         // per group: HD x 64 bf16
  static constexpr int LT = W + G * HD * 128;      // per group: local_out tile of the head, overwritten by dL
  static constexpr int DM = LT + G * TILE;         // per group: dmixed tile, overwritten by dR
  static constexpr int RED = DM + G * TILE;        // 4G warps x HD floats (dg_local partials)
  static constexpr int DSH = RED + 4 * G * HD * 4; // [max heads][128] gate grad ds per head and row
  static constexpr int CST = DSH + gate_max_heads<G>() * BM * 4;  // g_local, g_remote, then b_rout[h] per group
  static constexpr int BAR = CST + (2 + G) * HD * 4;
  static constexpr int BYTES = BAR + 256;
  static constexpr int THREADS = 64 + 128 * G;
  static constexpr int TMEM_COLS = G == 2 ? 512 : 256;
  static_assert(G == 2 || BYTES + 1024 <= 115 * 1024, "two CTAs per SM");
};

// per group g (0/1): W ready, R computed, dL/dR tiles ready, dlat MMA done,
// L/dmixed tiles loaded
enum { GB_W = 0, GB_R = 2, GB_DR = 4, GB_DL = 6, GB_F = 8, GB_NB = 10 };

// Warps: 0 = TMA producer (tiles in, dL/dR tiles out), 1 = TMEM + MMA issuer,
// 2-5 = group 0 (even heads), 6-9 = group 1 (odd heads); in a group thread =
// token row = TMEM lane.
//
// dg_remote needs no per-head reduction over R: with R_h = lat W_h^T + b_h,
//   dg_r = -sum_{t,h} ds R_h = -sum_h (S1_h W_h^T + S0_h b_h),
//   S1_h = sum_t ds[t,h] lat[t], S0_h = sum_t ds[t,h],
// formed from ds kept in shared memory after the head loop.
template <int HD, int G>
__global__ void __launch_bounds__(GbLayout<HD, G>::THREADS, G == 1 ? 2 : 1)
    gate_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_lo, const __grid_constant__ CUtensorMap tm_dm,
                       const __grid_constant__ CUtensorMap tm_dl, const __grid_constant__ CUtensorMap tm_dr,
                       Geom g, const bf16* __restrict__ lat, const bf16* __restrict__ w_rout,
                       const float* __restrict__ b_rout, const float* __restrict__ gl, const float* __restrict__ gr,
                       float* __restrict__ delta, float* __restrict__ dlat_tok, float* __restrict__ dg_part) {
  using L = GbLayout<HD, G>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + GB_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = blockIdx.y, t0 = blockIdx.x * BM;
  const int H = g.H;
  float* dsh = reinterpret_cast<float*>(smem + L::DSH);

  if (threadIdx.x == 0) LLATTN_TRACE_K(3, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < G; ++s) {
      mbar_init(&bars[GB_W + s], BM);
      mbar_init(&bars[GB_R + s], 1);
      mbar_init(&bars[GB_DR + s], BM);
      mbar_init(&bars[GB_DL + s], 1);
      mbar_init(&bars[GB_F + s], 1);
    }
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // R of group g at [g*HD, (g+1)*HD); dlat at G*128
  const uint32_t tDL = tmem + G * 128;
  float* red = reinterpret_cast<float*>(smem + L::RED);

  if (warp == 0) {
    // TMA producer. Head h uses group h%G's buffers; before loading head h
    // the producer stores head h-G's dL / dR tiles (written in place over the
    // local_out / dmixed tiles; 3-D (d, T, B) maps clip rows past T), waits
    // for its dlat MMA (reads dR) and for the stores to have read shared memory.
    if (lane == 0) {
      prefetch_tmap(&tm_lo);
      prefetch_tmap(&tm_dm);
      const int row0 = b * g.T + t0;
      int issued = 0;
      bool ok = true;
      auto store_head = [&](int h) -> bool {
        const int grp = h % G, n = h / G;
        if (!mbar_wait(&bars[GB_DR + grp], n & 1, abort, &g_fault_word)) return false;
#pragma unroll
        for (int p = 0; p < HD / 64; ++p) {
          tma_store_4d(&tm_dl, smem + L::LT + grp * L::TILE + p * (BM * 128), p * 64, h, t0, b);
          tma_store_4d(&tm_dr, smem + L::DM + grp * L::TILE + p * (BM * 128), p * 64, h, t0, b);
        }
        tma_store_commit();
        return true;
      };
      for (int h = 0; h < H; ++h) {
        const int grp = h % G, n = h / G;
        if (n >= 1) {
          if (!(ok = store_head(h - G))) break;
          if (!(ok = mbar_wait(&bars[GB_DL + grp], (n - 1) & 1, abort, &g_fault_word))) break;
          tma_store_wait_read();
        }
        if (h < 12) LLATTN_TRACE_K(3, 2 + h);
        mbar_expect_tx(&bars[GB_F + grp], 2 * L::TILE);
#pragma unroll
        for (int p = 0; p < HD / 64; ++p) {
          tma_load_4d(&tm_lo, &bars[GB_F + grp], smem + L::LT + grp * L::TILE + p * (BM * 128), p * 64, h, row0, 0);
          tma_load_4d(&tm_dm, &bars[GB_F + grp], smem + L::DM + grp * L::TILE + p * (BM * 128), p * 64, h, row0, 0);
        }
        issued = h + 1;
      }
      for (int h = H - G < 0 ? 0 : H - G; ok && h < H; ++h) ok = store_head(h);
      tma_store_wait_read();
      if (!ok) {
        raise_fault(g, kFaultProducer, abort);
        volatile int none = 0;
        volatile unsigned gnone = 0;
        for (int h = issued - G < 0 ? 0 : issued - G; h < issued; ++h)
          mbar_wait(&bars[GB_F + h % G], (h / G) & 1, &none, &gnone, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idR = idesc_bf16_f32(BM, HD, false, false);  // lat . W_h^T
      constexpr uint32_t idL = idesc_bf16_f32(BM, 64, false, true);   // dR_h . W_h
      const uint64_t dla = desc_sw128(smem_u32(smem + L::LAT), 16, 1024);
      bool ok = true;
      // head h belongs to group h&1 and is that group's (h>>1)-th head
      auto issue_r = [&](int h) -> bool {
        const int s = h % G;
        if (!mbar_wait(&bars[GB_W + s], (h / G) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint64_t dw = desc_sw128(smem_u32(smem + L::W + s * HD * 128), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(tmem + s * HD, desc_add(dla, kk * 32), desc_add(dw, kk * 32), idR, kk > 0);
        mma_commit(&bars[GB_R + s]);
        return true;
      };
      for (int x = 0; ok && x < G && x < H; ++x) ok = issue_r(x);
      for (int h = 0; ok && h < H; ++h) {
        const int s = h % G;
        if (!(ok = mbar_wait(&bars[GB_DR + s], (h / G) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint64_t dda = desc_sw128(smem_u32(smem + L::DM + s * L::TILE), 16, 1024);
        const uint64_t dwm = desc_sw128(smem_u32(smem + L::W + s * HD * 128), 0, 1024);
        // K steps past a padded head_dim would multiply zero-filled columns: skipped
#pragma unroll
        for (int kk = 0; kk < HD / 16 && kk * 16 < g.hd; ++kk)
          mma_bf16(tDL, desc_add(dda, (kk / 4) * (BM * 128) + (kk % 4) * 32), desc_add(dwm, kk * 2048), idL,
                   (h > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars[GB_DL + s]);
        if (h + G < H && !(ok = issue_r(h + G))) break;
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else if (warp >= 2) {
    const int grp = (warp - 2) >> 2;
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const int t = t0 + row;
    const bool valid = t < g.T;
    const int64_t tok = (int64_t)b * g.T + (valid ? t : 0);
    if (grp == 0) {  // lat row of this token, 128-byte swizzled rows
      const uint4* src = reinterpret_cast<const uint4*>(lat + ((int64_t)b * g.Tq + (valid ? t / g.qbs : 0)) * 64);
      uint8_t* d = smem + L::LAT + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(d + ((c ^ (row & 7)) * 16)) = src[c];
    }
    float* cgl = reinterpret_cast<float*>(smem + L::CST);  // g_local [HD], g_remote [HD]
    float* cbh = cgl + (2 + grp) * HD;                      // this group's b_rout[h]
    auto write_w = [&](int h) {  // into this group's W buffer, and b_rout[h]
      if (row < HD) {  // rows past a padded head_dim are zero
        const bool real = row < g.hd;
        const uint4* src = reinterpret_cast<const uint4*>(w_rout + ((int64_t)h * g.hd + (real ? row : 0)) * 64);
        uint8_t* d = smem + L::W + grp * HD * 128 + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(d + ((c ^ (row & 7)) * 16)) = real ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        cbh[row] = real ? b_rout[(int64_t)h * g.hd + row] : 0.f;
      }
      fence_async_smem();
      mbar_arrive(&bars[GB_W + grp]);
    };
    float* wred = red + (warp - 2) * HD;  // lane owns columns cc*32+lane
    for (int e = lane; e < HD; e += 32) wred[e] = 0.f;
    if (grp == 0 && row < HD) {
      cgl[row] = row < g.hd ? gl[row] : 0.f;
      cgl[HD + row] = row < g.hd ? gr[row] : 0.f;
    }
    bool ok = true;
    if (grp < H) write_w(grp);
    // tile rows: 16-byte chunk c of this row sits at panel c/8, slot (c%8)^(row%8)
    auto chunk_ptr = [&](uint8_t* tile, int c) -> uint4* {
      return reinterpret_cast<uint4*>(tile + (c >> 3) * (BM * 128) + row * 128 + (((c & 7) ^ (row & 7)) * 16));
    };
    for (int h = grp; h < H; h += G) {
      const int n = h / G;  // this group's n-th head
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_R + grp], n & 1, abort, &g_fault_word));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_F + grp], n & 1, abort, &g_fault_word));
      if (!ok) break;
      if (row == 0 && h < 12) LLATTN_TRACE_K(3, 14 + h);
      tc_fence_after();
      const uint32_t tR = tmem + grp * HD + lane_off;
      uint8_t* lt = smem + L::LT + grp * L::TILE;
      uint8_t* dmt = smem + L::DM + grp * L::TILE;
      // b_rout[h] (and at the first head the gate vectors), written by the
      // group's threads before they arrived on GB_W: that phase completing
      // publishes them (a bounded wait, unlike a named barrier)
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_W + grp], n & 1, abort, &g_fault_word));
      if (!ok) break;
      const float4* bh4 = reinterpret_cast<const float4*>(cbh);
      const float4* gl4 = reinterpret_cast<const float4*>(cgl);
      const float4* gr4 = reinterpret_cast<const float4*>(cgl + HD);
      // pass 1: gate logits and dw, two columns per f32x2 operation
      uint64_t sl2 = 0, sr2 = 0, dw2 = 0;
#pragma unroll 1
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t rr[32];
        tmem_ld32(tR + cc * 32, rr);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 lq = *chunk_ptr(lt, cc * 4 + q), mq = *chunk_ptr(dmt, cc * 4 + q);
          const uint32_t lw[4] = {lq.x, lq.y, lq.z, lq.w}, mw[4] = {mq.x, mq.y, mq.z, mq.w};
#pragma unroll
          for (int i4 = 0; i4 < 2; ++i4) {
            const int c4 = (cc * 32 + q * 8) / 4 + i4;
            const float4 bb = bh4[c4], ga = gl4[c4], gb = gr4[c4];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int pi = i4 * 2 + k;  // column pair within the chunk
              const uint64_t l2 = bf2_to_f2(lw[pi]), m2 = bf2_to_f2(mw[pi]);
              const uint64_t r2 = f2_add(f2_pack(__uint_as_float(rr[q * 8 + 2 * pi]), __uint_as_float(rr[q * 8 + 2 * pi + 1])),
                                         k ? f2_pack(bb.z, bb.w) : f2_pack(bb.x, bb.y));
              sl2 = f2_fma(l2, k ? f2_pack(ga.z, ga.w) : f2_pack(ga.x, ga.y), sl2);
              sr2 = f2_fma(r2, k ? f2_pack(gb.z, gb.w) : f2_pack(gb.x, gb.y), sr2);
              dw2 = f2_fma(m2, f2_sub(l2, r2), dw2);
            }
          }
        }
      }
      if (row == 0 && h < 12) LLATTN_TRACE_K(3, 26 + h);
      float sla, slb, sra, srb, dwa, dwb;
      f2_unpack(sl2, sla, slb);
      f2_unpack(sr2, sra, srb);
      f2_unpack(dw2, dwa, dwb);
      const float x = (sla + slb) + g.gate_bias - (sra + srb);
      const float w = 1.f / (1.f + expf(-x));
      const float wr = 1.f / (1.f + expf(x));
      const float ds = valid ? (dwa + dwb) * w * wr : 0.f;
      dsh[h * BM + row] = ds;
      // pass 2: dL over local_out and dR over dmixed in the tiles (same
      // thread, same bytes, after reading them), D = dL.L, dg_local partial.
      // Rows past T (the next sequence's rows in the 2-D load) have ds = 0
      // and their dL / dR are clipped by the 3-D store maps.
      const uint64_t w2 = f2_pack(w, w), wr2 = f2_pack(wr, wr), ds2 = f2_pack(ds, ds), nds2 = f2_pack(-ds, -ds);
      uint64_t dsum2 = 0;
#pragma unroll 1
      for (int cc = 0; cc < HD / 32; ++cc) {
        float al[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4* lp = chunk_ptr(lt, cc * 4 + q);
          uint4* mp = chunk_ptr(dmt, cc * 4 + q);
          const uint4 lq = *lp, mq = *mp;
          const uint32_t lw[4] = {lq.x, lq.y, lq.z, lq.w}, mw[4] = {mq.x, mq.y, mq.z, mq.w};
          uint32_t pdl[4], pdr[4];
#pragma unroll
          for (int i4 = 0; i4 < 2; ++i4) {
            const int c4 = (cc * 32 + q * 8) / 4 + i4;
            const float4 ga = gl4[c4], gb = gr4[c4];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int pi = i4 * 2 + k;
              const uint64_t l2 = bf2_to_f2(lw[pi]), m2 = bf2_to_f2(mw[pi]);
              const uint64_t dl2 = f2_fma(w2, m2, f2_mul(ds2, k ? f2_pack(ga.z, ga.w) : f2_pack(ga.x, ga.y)));
              const uint64_t dr2 = f2_fma(wr2, m2, f2_mul(nds2, k ? f2_pack(gb.z, gb.w) : f2_pack(gb.x, gb.y)));
              float a0, a1, r0, r1;
              f2_unpack(dl2, a0, a1);
              f2_unpack(dr2, r0, r1);
              pdl[pi] = pack_bf16(a0, a1);
              pdr[pi] = pack_bf16(r0, r1);
              // D from the stored (bf16-rounded) dL
              dsum2 = f2_fma(bf2_to_f2(pdl[pi]), l2, dsum2);
              f2_unpack(f2_mul(ds2, l2), al[q * 8 + 2 * pi], al[q * 8 + 2 * pi + 1]);
            }
          }
          *lp = make_uint4(pdl[0], pdl[1], pdl[2], pdl[3]);
          *mp = make_uint4(pdr[0], pdr[1], pdr[2], pdr[3]);
        }
        wred[cc * 32 + lane] += butterfly32(al, lane);
      }
      float dsa, dsb;
      f2_unpack(dsum2, dsa, dsb);
      const float dsum = dsa + dsb;
      if (valid) delta[((int64_t)b * H + h) * g.T + t] = dsum;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[GB_DR + grp]);
      if (row == 0 && h < 12) LLATTN_TRACE_K(3, 38 + h);
      // W buffer reuse: the dlat MMA of head h must have read it
      if (h + G < H) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_DL + grp], n & 1, abort, &g_fault_word));
        if (!ok) break;
        if (row == 0 && h < 10) LLATTN_TRACE_K(3, 50 + h);
        write_w(h + G);
      }
    }
    if (!ok) raise_fault(g, kFaultSoftmax, abort);
    if (grp == 0) {
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_DL + ((H - 1) % G)], ((H - 1) / G) & 1, abort,
                                                     &g_fault_word));
      if (!ok) {
        raise_fault(g, kFaultEpilogue, abort);
      } else {
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t r[32];
          tmem_ld32(tDL + lane_off + cc * 32, r);
          tmem_ld_wait();
          if (valid) {
            float4* d = reinterpret_cast<float4*>(dlat_tok + tok * 64 + cc * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              d[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                 __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) LLATTN_TRACE_K(3, 60);
  const int64_t part = ((int64_t)b * gridDim.x + blockIdx.x) * gate_dg_stride(g.hd, H);
  // dg_local partial [cta][0, HD): summed over the compute warps
  for (int e = threadIdx.x; e < g.hd; e += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < 4 * G; ++w8) v += red[w8 * HD + e];
    dg_part[part + e] = v;
  }
  // dg_remote is linear in S1_h[e] = sum_rows ds lat[row, e] and
  // S0_h = sum_rows ds: their per-CTA partials go to [cta][HD + h*65 + e]
  // (e = 64: S0) and gate_dgr_finalize_kernel applies W_h, b_h once to the
  // sums. Thread = (head, 4 consecutive e), 4 independent accumulators.
  const bool all_ok = !*abort;
  for (int idx = threadIdx.x; idx < H * 16; idx += blockDim.x) {
    const int h = idx >> 4, e0 = (idx & 15) * 4;
    const int c = e0 >> 3, k0 = (e0 & 7) * 2;  // 16-byte chunk, byte offset in it
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, s0 = 0.f;
    if (all_ok) {
      const float* dh = dsh + h * BM;
#pragma unroll 8
      for (int r = 0; r < BM; ++r) {
        const uint2 lv = *reinterpret_cast<const uint2*>(smem + L::LAT + r * 128 + ((c ^ (r & 7)) * 16) + k0);
        const float dsv = dh[r];
        const float2 l01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lv.x));
        const float2 l23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lv.y));
        a0 = fmaf(dsv, l01.x, a0);
        a1 = fmaf(dsv, l01.y, a1);
        a2 = fmaf(dsv, l23.x, a2);
        a3 = fmaf(dsv, l23.y, a3);
        s0 += dsv;
      }
    }
    float* o = dg_part + part + g.hd + h * 65;
    o[e0] = a0;  // rows of 65 floats: not 16-byte aligned
    o[e0 + 1] = a1;
    o[e0 + 2] = a2;
    o[e0 + 3] = a3;
    if (e0 == 0) o[64] = s0;
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------

constexpr int DW_ST = 4;  // pipeline stages of 64 tokens

struct DwLayout {
  static constexpr int A = 0;                    // DW_ST x (64 tokens x 128 cols bf16) = 16 KB each
  static constexpr int B = A + DW_ST * 16384;    // DW_ST x (64 tokens x 64 bf16) = 8 KB each
  static constexpr int ONES = B + DW_ST * 8192;  // 16 x 64 bf16 ones: B operand of the column-sum MMA
  static constexpr int BAR = ONES + 2048;
  static constexpr int BYTES = BAR + 256;
};

enum { DW_FA = 0, DW_FB = DW_ST, DW_E = 2 * DW_ST, DW_DONE = 3 * DW_ST, DW_NB = 3 * DW_ST + 1 };

// dW partial [128 columns of d x 64] over this split's tokens, and db as a
// second MMA against a ones tile (D2[:, j] = sum over tokens of dR, for
// every j): the tensor pipe does both reductions. Token-wise queries
// (qbs = 1): the lat rows of a 64-token chunk are one TMA box; block-pooled
// ones are gathered by the threads.
__global__ void __launch_bounds__(192, 2)
    rout_dw_tc_kernel(const __grid_constant__ CUtensorMap tm_dr, const __grid_constant__ CUtensorMap tm_lat, Geom g,
                      const bf16* __restrict__ lat, float* __restrict__ dw_part, float* __restrict__ db_part,
                      int n_split) {
  using L = DwLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + DW_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c0 = blockIdx.x * 128, split = blockIdx.y;
  const int n_tok = g.B * g.T;
  // split boundaries are multiples of 64 tokens; the last chunk's rows past
  // n_tok are zero-filled by the copies (or zeroed by the gathering threads)
  const int per = cdiv(cdiv(n_tok, n_split), 64) * 64;
  const int na = split * per, nb = min(n_tok, na + per);
  const int nch = nb > na ? cdiv(nb - na, 64) : 0;
  const bool lat_tma = g.qbs == 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < DW_ST; ++s) {
      mbar_init(&bars[DW_FA + s], 1);
      mbar_init(&bars[DW_FB + s], 128);
      mbar_init(&bars[DW_E + s], 1);
    }
    mbar_init(&bars[DW_DONE], 1);
    *abort = 0;
    fence_barrier_init();
  }
  {  // ones tile, K-major 128-byte-swizzled (every element 1.0, so the swizzle is moot)
    uint4* o = reinterpret_cast<uint4*>(smem + L::ONES);
    for (int i = threadIdx.x; i < 2048 / 16; i += blockDim.x) o[i] = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    fence_async_smem();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // dW partial at [0, 64), column sums at [64, 80)

  if (warp == 0) {
    if (lane == 0 && nch > 0) {
      prefetch_tmap(&tm_dr);
      if (lat_tma) prefetch_tmap(&tm_lat);
      int issued = 0;
      for (int i = 0; i < nch; ++i) {
        const int s = i % DW_ST;
        if (i >= DW_ST && !mbar_wait(&bars[DW_E + s], ((i / DW_ST) - 1) & 1, abort, &g_fault_word)) {
          raise_fault(g, kFaultProducer, abort);
          break;
        }
        mbar_expect_tx(&bars[DW_FA + s], 16384 + (lat_tma ? 8192 : 0));
        tma_load_2d(&tm_dr, &bars[DW_FA + s], smem + L::A + s * 16384, c0, na + i * 64);
        tma_load_2d(&tm_dr, &bars[DW_FA + s], smem + L::A + s * 16384 + 8192, c0 + 64, na + i * 64);
        if (lat_tma) tma_load_2d(&tm_lat, &bars[DW_FA + s], smem + L::B + s * 8192, 0, na + i * 64);
        issued = i + 1;
      }
      if (*abort) {
        volatile int none = 0;
        volatile unsigned gnone = 0;
        for (int i = issued - DW_ST < 0 ? 0 : issued - DW_ST; i < issued; ++i)
          mbar_wait(&bars[DW_FA + i % DW_ST], (i / DW_ST) & 1, &none, &gnone, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nch > 0) {
      constexpr uint32_t id = idesc_bf16_f32(128, 64, true, true);
      constexpr uint32_t id1 = idesc_bf16_f32(128, 16, true, false);
      const uint64_t d1 = desc_sw128(smem_u32(smem + L::ONES), 16, 1024);
      bool ok = true;
      for (int i = 0; ok && i < nch; ++i) {
        const int s = i % DW_ST;
        if (!(ok = mbar_wait(&bars[DW_FA + s], (i / DW_ST) & 1, abort, &g_fault_word))) break;
        if (!lat_tma && !(ok = mbar_wait(&bars[DW_FB + s], (i / DW_ST) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint64_t da = desc_sw128(smem_u32(smem + L::A + s * 16384), 8192, 1024);
        const uint64_t db = desc_sw128(smem_u32(smem + L::B + s * 8192), 0, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          mma_bf16(tmem, desc_add(da, kk * 2048), desc_add(db, kk * 2048), id, acc);
          mma_bf16(tmem + 64, desc_add(da, kk * 2048), desc_add(d1, kk * 32), id1, acc);
        }
        mma_commit(&bars[DW_E + s]);
      }
      mma_commit(&bars[DW_DONE]);
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    const int tid = threadIdx.x - 64;  // 0..127
    bool ok = true;
    if (!lat_tma) {
      for (int i = 0; i < nch; ++i) {
        const int s = i % DW_ST;
        if (i >= DW_ST) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bars[DW_E + s], ((i / DW_ST) - 1) & 1, abort, &g_fault_word));
          if (!ok) break;
        }
        // B tile: 64 token rows of lat (row r of token n = b*T + t -> lat row b*Tq + t/qbs)
        const int r = tid >> 1, half = tid & 1;
        const int n = na + i * 64 + r;
        uint8_t* d = smem + L::B + s * 8192 + r * 128;
        if (n < nb) {
          const int bb = n / g.T, tt = n % g.T;
          const uint4* src = reinterpret_cast<const uint4*>(lat + ((int64_t)bb * g.Tq + tt / g.qbs) * 64);
#pragma unroll
          for (int c = half * 4; c < half * 4 + 4; ++c) *reinterpret_cast<uint4*>(d + ((c ^ (r & 7)) * 16)) = src[c];
        } else {
#pragma unroll
          for (int c = half * 4; c < half * 4 + 4; ++c)
            *reinterpret_cast<uint4*>(d + ((c ^ (r & 7)) * 16)) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_async_smem();
        mbar_arrive(&bars[DW_FB + s]);
      }
      if (!ok) raise_fault(g, kFaultSoftmax, abort);
    }
    if (ok && nch > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars[DW_DONE], 0, abort, &g_fault_word));
    if (!ok) {
      raise_fault(g, kFaultEpilogue, abort);
    } else {
      tc_fence_after();
      const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
      const int m = 32 * (warp & 3) + lane;  // TMEM lane = output row (column of d)
      float* dst = dw_part + (int64_t)split * g.d * 64 + (int64_t)(c0 + m) * 64;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        if (nch > 0) {
          tmem_ld32(tmem + lane_off + cc * 32, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) r[q] = 0u;
        }
        if (c0 + m < g.d) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<float4*>(dst + cc * 32)[q] = make_float4(
                __uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                __uint_as_float(r[4 * q + 3]));
        }
      }
      uint32_t r1[16];
      if (nch > 0) {
        tmem_ld16(tmem + lane_off + 64, r1);
        tmem_ld_wait();
      } else {
        r1[0] = 0u;
      }
      if (c0 + m < g.d) db_part[(int64_t)split * g.d + c0 + m] = __uint_as_float(r1[0]);
      (void)tid;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// dlat rows of block-pooled queries: dlat[b, r] = sum of dlat_tok over the
// row's tokens (token-wise queries use dlat_tok directly).
__global__ void dlat_rowsum_kernel(Geom g, const float* __restrict__ dlat_tok, float* __restrict__ dlat) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)g.B * g.Tq * 64) return;
  const int e = i % 64;
  const int64_t br = i / 64;
  const int b = br / g.Tq, r = br % g.Tq;
  float a = 0.f;
  for (int t = r * g.qbs; t < min(g.T, (r + 1) * g.qbs); ++t) a += dlat_tok[((int64_t)b * g.T + t) * 64 + e];
  dlat[i] = a;
}
