// Forward of the tensor-core local branch, two query tiles per CTA
// ("ping-pong"; included by local_sm100.cu).
//
// One CTA per (batch, head, 256 queries) = query tiles A (rows q0..q0+127)
// and B (q0+128..q0+255); 10 warps:
//   warp 0     TMA producer: Q_A, Q_B, then the 64-key K/V tiles of the union
//              of both tiles' key ranges, in a 2-stage ring (a key tile in
//              the overlap is loaded once for both)
//   warp 1     TMEM allocator (512 columns) and single-thread MMA issuer. For
//              each key tile: S_A, S_B of the next tile, then PV_A, PV_B of
//              this one, so one group's softmax overlaps the other's MMAs.
//              After a group's last PV, its remote tile R = lat W_h^T goes
//              into that group's freed S columns.
//   warps 2-5  softmax of tile A, warps 6-9 softmax of tile B: thread = query
//              row = TMEM lane; online softmax with the window mask, P bf16
//              written back over the S columns it came from (the PV MMA
//              reads it from TMEM), O rescale in TMEM, fused gate epilogue.
// TMEM: S_A x2 [0,128), S_B x2 [128,256), O_A [256,256+hd), O_B after it.
// Shared memory: Q_A, Q_B, the K/V ring, and per group the remote-tile
// operands (lat rows, a copy of the head's W_rout slice) written at kernel
// start; in the epilogue local_out is staged over the group's Q tile and
// mixed over its remote-operand region, so the groups never wait for each
// other.

// PAIR: two query tiles per CTA (ping-pong), 512 TMEM columns, one CTA per SM.
// !PAIR: one query tile per CTA, 256 TMEM columns and under 113 KB of shared
// memory, two CTAs per SM: one CTA's prologue and epilogue overlap the other's
// main loop. The remote-tile operands then overlay the Q tile once its S MMAs
// are done (hd 128), and the epilogue stages local_out / mixed over the K / V
// ring.
template <int HD, bool PAIR = true>
struct FwdPPLayout {
  static constexpr int BNK = 64;
  static constexpr int QPANEL = BM * 128;
  static constexpr int KPANEL = BNK * 128;
  static constexpr int QTILE = BM * HD * 2;
  static constexpr int KTILE = BNK * HD * 2;
  static constexpr int QA = 0;
  static constexpr int QB = PAIR ? QA + QTILE : QA;
  static constexpr int NST = PAIR ? 3 : 2;      // K/V ring depth
  static constexpr int K = QB + QTILE;          // NST stages (QB = QA without PAIR)
  static constexpr int V = K + NST * KTILE;     // NST stages
  // per group x at X + x * XS: lat rows (128 x 64 bf16) then W_rout[h] (hd x 64)
  static constexpr int XS = BM * 128 + HD * 128;
  static constexpr bool X_OVER_Q = !PAIR && XS <= QTILE;
  static constexpr int X = X_OVER_Q ? QA : V + NST * KTILE;
  static constexpr int CST = X_OVER_Q ? V + NST * KTILE : X + (PAIR ? 2 : 1) * XS;
  static constexpr int BAR = CST + 3 * HD * 4;  // b_rout[h], g_local, g_remote (hd floats each)
  static constexpr int BYTES = BAR + 320;  // PP_NB barriers, TMEM slot, abort flag
  static constexpr int TMEM_COLS = PAIR ? 512 : 256;
  static constexpr int O_BASE = PAIR ? 256 : 128;  // O_x at O_BASE + x * hd
  static constexpr int THREADS = PAIR ? 320 : 192;
  static_assert(!PAIR || XS >= QTILE, "mixed tile staged over the remote operands");
  static_assert(PAIR || NST * KTILE >= QTILE, "local_out / mixed staged over the K / V ring");
  static_assert(PAIR || BYTES + 1024 <= 113 * 1024, "two CTAs per SM");
};

// per group g: S[2], P[2] (softmax arrivals), O[2] (PV done) — one barrier
// per buffer, so a group running a tile ahead never makes a parity wait
// ambiguous — plus LW (remote operands written) and R; shared: Q, K / V
// loaded and K / V stage free per ring stage
enum {
  PP_Q = 0, PP_K = 1, PP_V = 4, PP_VE = 7,  // K, V loaded, V stage free: + stage (3)
  PP_LW = 10,  // + g
  PP_S = 12,   // + 2*g + buffer
  PP_P = 16,   // + 2*g + buffer
  PP_O = 20,   // + 2*g + buffer
  PP_R = 24,   // + g
  PP_EP = 26,  // + g: epilogue tiles staged
  PP_SD = 28,  // group A's S MMAs done (!PAIR: Q free for the remote operands)
  PP_KE = 29,  // + stage (3): K stage free (its tile's S MMAs done)
  PP_NB = 32
};

// The running max of a row is only moved (and O rescaled) when the new
// maximum exceeds it by more than this many powers of two; otherwise P uses
// the stale max and stays below 2^kRescaleLog2.
constexpr float kRescaleLog2 = 8.f;

struct PPTiles {
  int first, last;  // key-tile range [first, last] of a query tile; last < first: none
  __device__ bool has(int j) const { return j >= first && j <= last; }
  __device__ int n() const { return last >= first ? last - first + 1 : 0; }
};

template <int HD, bool PAIR>
__global__ void __launch_bounds__(FwdPPLayout<HD, PAIR>::THREADS, PAIR ? 1 : 2)
    local_fwd_pp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv,
                        const __grid_constant__ CUtensorMap tm_lo, const __grid_constant__ CUtensorMap tm_mx,
                        const __grid_constant__ CUtensorMap tm_lat, const __grid_constant__ CUtensorMap tm_w, Geom g,
                        bf16* __restrict__ local_out, float* __restrict__ lse_out, GateEpilogue ep) {
  using L = FwdPPLayout<HD, PAIR>;
  constexpr int BNK = L::BNK;
  extern __shared__ __align__(1024) uint8_t smem_pp[];
  uint8_t* smem = smem_pp;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + PP_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) raise_fault(g, kFaultEpilogue, nullptr);
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // heads fastest: CTAs that run together cover whole token rows of qkv
  const int h = blockIdx.x, b = blockIdx.z;
  const int q0 = blockIdx.y * (PAIR ? 2 : 1) * BM;
  if (threadIdx.x == 0) LLATTN_TRACE_K(1, 0);
  const bool fuse = ep.lat != nullptr;
  const bool has_b = PAIR && q0 + BM < g.T;
  const int kbase = local_lo(g, q0);  // first key of the union range
  // key tiles [kbase + 64 j, +64) used by each query tile
  PPTiles tA, tB;
  {
    const int lastA = min(q0 + BM - 1, g.T - 1) - 1;  // last key of tile A
    tA.first = 0;
    tA.last = lastA >= kbase ? (lastA - kbase) / BNK : -1;
    if (has_b) {
      const int loB = local_lo(g, q0 + BM), lastB = min(q0 + 2 * BM - 1, g.T - 1) - 1;
      tB.first = (loB - kbase) / BNK;
      tB.last = lastB >= loB ? (lastB - kbase) / BNK : -1;
    } else {
      tB.first = 0;
      tB.last = -1;
    }
  }
  const int nk = max(tA.last, tB.last) + 1;

  if (threadIdx.x == 0) {
    mbar_init(&bars[PP_Q], 1);
    for (int s = 0; s < L::NST; ++s) {
      mbar_init(&bars[PP_K + s], 1);
      mbar_init(&bars[PP_V + s], 1);
      mbar_init(&bars[PP_VE + s], 1);
      mbar_init(&bars[PP_KE + s], 1);
    }
    for (int x = 0; x < 4; ++x) {
      mbar_init(&bars[PP_S + x], 1);
      mbar_init(&bars[PP_P + x], BM);
      mbar_init(&bars[PP_O + x], 1);
    }
    mbar_init(&bars[PP_SD], 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars[PP_LW + x], BM + 1);
      mbar_init(&bars[PP_R + x], 1);
      mbar_init(&bars[PP_EP + x], BM);
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
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) LLATTN_TRACE_K(1, 1);

  if (warp == 0) {
    if (lane == 0 && (nk > 0 || fuse)) {
      int issued = 0;
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_kv);
      auto load_remote = [&]() {
        // remote-tile operands: W_rout[h] for each group, the lat rows of
        // token-wise queries (block-pooled ones are written by the threads),
        // and the epilogue's per-column constants (with group A's barrier)
        const bool lat_tma = g.qbs == 1;
#pragma unroll
        for (int x = 0; x < (PAIR ? 2 : 1); ++x) {
          uint8_t* xr = smem + L::X + x * L::XS;
          mbar_expect_tx(&bars[PP_LW + x], HD * 128 + (lat_tma ? BM * 128 : 0) + (x == 0 ? 3 * g.hd * 4 : 0));
          tma_load_2d(&tm_w, &bars[PP_LW + x], xr + BM * 128, 0, h * g.hd);
          if (lat_tma) tma_load_3d(&tm_lat, &bars[PP_LW + x], xr, 0, q0 + x * BM, b);
        }
        float* cst = reinterpret_cast<float*>(smem + L::CST);
        bulk_load(cst, ep.b_rout + (int64_t)h * g.hd, g.hd * 4, &bars[PP_LW + 0]);
        bulk_load(cst + HD, ep.g_local, g.hd * 4, &bars[PP_LW + 0]);
        bulk_load(cst + 2 * HD, ep.g_remote, g.hd * 4, &bars[PP_LW + 0]);
      };
      if (fuse && !L::X_OVER_Q) load_remote();
      if (nk > 0) {
        mbar_expect_tx(&bars[PP_Q], (PAIR ? 2 : 1) * L::QTILE);
        tma_load_tile<HD / 64, BM>(&tm_q, &bars[PP_Q], smem + L::QA, q0, h, b);
        if (PAIR) tma_load_tile<HD / 64, BM>(&tm_q, &bars[PP_Q], smem + L::QB, q0 + BM, h, b);
      }
      // K stages free once their tile's S MMAs are done, V stages once its
      // PV MMAs are: K tiles are issued one tile ahead of V tiles, so a K
      // load never waits behind a PV
      int issued_v = 0;
      auto load_kv = [&](int j, bool is_k) -> bool {
        const int s = j % L::NST;
        if (j >= L::NST &&
            !mbar_wait(&bars[(is_k ? PP_KE : PP_VE) + s], ((j / L::NST) - 1) & 1, abort, &g_fault_word))
          return false;
        const int bar = (is_k ? PP_K : PP_V) + s;
        mbar_expect_tx(&bars[bar], L::KTILE);
        tma_load_tile<HD / 64, BNK>(&tm_kv, &bars[bar], smem + (is_k ? L::K : L::V) + s * L::KTILE, kbase + j * BNK,
                      (is_k ? 1 : 2) * g.H + h, b);
        if (is_k) issued = j + 1; else issued_v = j + 1;
        return true;
      };
      for (int j = 0; j <= nk; ++j) {
        if ((j < nk && !load_kv(j, true)) || (j >= 1 && !load_kv(j - 1, false))) {
          raise_fault(g, kFaultProducer, abort);
          break;
        }
      }
      if (fuse && L::X_OVER_Q && !*abort) {  // the remote operands go over Q once its S MMAs are done
        if (mbar_wait(&bars[PP_SD], 0, abort, &g_fault_word))
          load_remote();
        else
          raise_fault(g, kFaultProducer, abort);
      }
      if (*abort) {
        // let the copies already issued land before the CTA can exit
        volatile int none = 0;
        volatile unsigned gnone = 0;
        if (nk > 0) mbar_wait(&bars[PP_Q], 0, &none, &gnone, 100000000ull);
        if (fuse)
          for (int x = 0; x < (PAIR ? 2 : 1); ++x) mbar_wait(&bars[PP_LW + x], 0, &none, &gnone, 100000000ull);
        for (int j = issued - L::NST < 0 ? 0 : issued - L::NST; j < issued; ++j)
          mbar_wait(&bars[PP_K + j % L::NST], (j / L::NST) & 1, &none, &gnone, 100000000ull);
        for (int j = issued_v - L::NST < 0 ? 0 : issued_v - L::NST; j < issued_v; ++j)
          mbar_wait(&bars[PP_V + j % L::NST], (j / L::NST) & 1, &none, &gnone, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BNK, false, false);
      constexpr uint32_t idO = idesc_bf16_f32(BM, HD, false, true);
      constexpr uint32_t idR = idesc_bf16_f32(BM, HD, false, false);
      const uint64_t dqa0 = desc_sw128(smem_u32(smem + L::QA), 16, 1024);
      const uint64_t dqb0 = desc_sw128(smem_u32(smem + L::QB), 16, 1024);
      bool ok = true;
      // Event-driven issue: each pass tests (without blocking) what has
      // become ready and issues it, so neither group waits for the other.
      //   S_x(i): K tile loaded, and S buffer i&1 free: PV_x(i-2), which
      //           reads P_x(i-2) from those columns, issued (i <= npv + 1)
      //   PV_x(i): P_x(i) landed and V tile loaded
      //   R_x: after the group's last PV, once its lat / W_rout rows are in
      // A K stage is released (KE commit) once every group using the tile has
      // issued its S for it, a V stage (VE) once they have issued its PV;
      // releases happen in tile order.
      int ns[2] = {0, 0}, npv[2] = {0, 0};
      bool r_done[2] = {false, false};
      const int nx[2] = {tA.n(), has_b ? tB.n() : 0};
      const int first[2] = {tA.first, tB.first};
      const bool grp_on[2] = {true, has_b};
      int released = 0, k_released = 0;  // tiles whose V / K stage was released
      if (nk > 0) ok = mbar_wait(&bars[PP_Q], 0, abort, &g_fault_word);
      LLATTN_TRACE_K(1, 2);
      uint64_t t_last = globaltimer_ns();
      uint32_t spin = 0;
      bool sd_done = false;
      while (ok) {
        bool progress = false, all_done = true;
        if (!sd_done && ns[0] == nx[0]) {  // group A's S MMAs all issued: Q_A free once they complete
          mma_commit(&bars[PP_SD]);
          sd_done = true;
        }
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (!grp_on[x]) continue;
          // S
          if (ns[x] < nx[x] && ns[x] <= npv[x] + 1) {
            const int j = first[x] + ns[x], st = j % L::NST;
            if (mbar_test_wait(&bars[PP_K + st], (j / L::NST) & 1)) {
              tc_fence_after();
              const uint64_t dka = desc_sw128(smem_u32(smem + L::K + st * L::KTILE), 16, 1024);
              const uint32_t dst = tmem + x * 128 + (ns[x] & 1) * BNK;
              const uint64_t dqa = x ? dqb0 : dqa0;
              // K steps past a padded head_dim would multiply zero-filled columns: skipped
#pragma unroll
              for (int kk = 0; kk < HD / 16 && kk * 16 < g.hd; ++kk)
                mma_bf16(dst, desc_add(dqa, (kk / 4) * L::QPANEL + (kk % 4) * 32),
                         desc_add(dka, (kk / 4) * L::KPANEL + (kk % 4) * 32), idS, kk > 0);
              mma_commit(&bars[PP_S + 2 * x + (ns[x] & 1)]);
              ++ns[x];
              progress = true;
            }
          }
          // PV
          if (npv[x] < ns[x]) {
            const int i = npv[x], j = first[x] + i, st = j % L::NST;
            if (mbar_test_wait(&bars[PP_P + 2 * x + (i & 1)], (i >> 1) & 1) &&
                mbar_test_wait(&bars[PP_V + st], (j / L::NST) & 1)) {
              tc_fence_after();
              // P (bf16, packed two per column) over the first 32 columns of S buffer i&1
              const uint32_t pa = tmem + x * 128 + (i & 1) * BNK, to = tmem + L::O_BASE + x * HD;
              const uint64_t dva = desc_sw128(smem_u32(smem + L::V + st * L::KTILE), L::KPANEL, 1024);
#pragma unroll
              for (int kk = 0; kk < BNK / 16; ++kk)
                mma_bf16_ts(to, pa + kk * 8, desc_add(dva, kk * 2048), idO, (i > 0 || kk > 0) ? 1u : 0u);
              mma_commit(&bars[PP_O + 2 * x + (i & 1)]);
              ++npv[x];
              progress = true;
            }
          }
          // R
          if (fuse && !r_done[x] && npv[x] == nx[x]) {
            if (mbar_test_wait(&bars[PP_LW + x], 0)) {
              tc_fence_after();
              const uint32_t la = smem_u32(smem + L::X + x * L::XS);
              const uint64_t dla = desc_sw128(la, 16, 1024), dwa = desc_sw128(la + BM * 128, 16, 1024);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_bf16(tmem + x * 128, desc_add(dla, kk * 32), desc_add(dwa, kk * 32), idR, kk > 0);
              mma_commit(&bars[PP_R + x]);
              r_done[x] = true;
              progress = true;
            }
          }
          if (npv[x] < nx[x] || (fuse && !r_done[x])) all_done = false;
        }
        // release K stages in tile order once every group using the tile
        // has issued its S MMAs, V stages once they have issued their PV
        while (k_released < nk) {
          const int j = k_released;
          bool used_done = true;
#pragma unroll
          for (int x = 0; x < 2; ++x)
            if (grp_on[x] && j >= first[x] && j < first[x] + nx[x] && ns[x] <= j - first[x]) used_done = false;
          if (!used_done) break;
          mma_commit(&bars[PP_KE + j % L::NST]);
          ++k_released;
          progress = true;
        }
        while (released < nk) {
          const int j = released;
          bool used_done = true;
#pragma unroll
          for (int x = 0; x < 2; ++x)
            if (grp_on[x] && j >= first[x] && j < first[x] + nx[x] && npv[x] <= j - first[x]) used_done = false;
          if (!used_done) break;
          mma_commit(&bars[PP_VE + j % L::NST]);
          ++released;
          progress = true;
        }
        if (all_done && released == nk && k_released == nk) break;
        if (progress) {
          t_last = globaltimer_ns();
          spin = 0;
        } else if ((++spin & 63u) == 0) {
          if (*abort || g_fault_word || globaltimer_ns() - t_last > 1000000000ull) ok = false;
        }
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    const int grp = (warp - 2) >> 2;  // 0: tile A, 1: tile B
    const PPTiles tt = grp ? tB : tA;
    const int n_mine = tt.n();
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const int t = q0 + grp * BM + row;
    const bool valid = t < g.T;
    const int lo = valid ? local_lo(g, t) : 0x7fffffff;
    const float sc = g.scale * kLog2e;
    float m = -INFINITY, l = 0.f;  // m: reference max (log2 domain) of P and O
    const uint32_t tS = tmem + grp * 128, tO = tmem + L::O_BASE + grp * HD, tR = tmem + grp * 128;
    uint8_t* xreg = smem + L::X + grp * L::XS;  // this group's lat rows, then W_rout[h]
    float* cst = reinterpret_cast<float*>(smem + L::CST);
    bool ok = true;
    // block-pooled latent queries: this row's lat row (token-wise ones and
    // W_rout come by TMA); with the operands over Q, after its S MMAs
    auto write_lat_rows = [&]() {
      // padded head_dim: the per-column constants past hd are zero (the bulk
      // copies bring hd of them), so padded columns add nothing to the logits
      if (grp == 0 && row < HD - g.hd) {
        cst[g.hd + row] = 0.f;
        cst[HD + g.hd + row] = 0.f;
        cst[2 * HD + g.hd + row] = 0.f;
      }
      if (g.qbs != 1) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const bf16*>(ep.lat) +
                                                          ((int64_t)b * g.Tq + (valid ? t / g.qbs : 0)) * 64);
        uint8_t* dl_ = xreg + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dl_ + ((c ^ (row & 7)) * 16)) = src[c];
        fence_async_smem();
      }
      mbar_arrive(&bars[PP_LW + grp]);
    };
    if (fuse && !L::X_OVER_Q) write_lat_rows();
    if (!(grp == 1 && !has_b)) {
      const uint64_t sc2 = f2_pack(sc, sc);
      for (int i = 0; ok && i < n_mine; ++i) {
        const int j = tt.first + i;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[PP_S + 2 * grp + (i & 1)], (i >> 1) & 1, abort, &g_fault_word));
        if (!ok) break;
        if (row == 0) LLATTN_TRACE_K(1, 4 + grp * 24 + i);
        tc_fence_after();
        const uint32_t tsrc = tS + (i & 1) * BNK + lane_off;
        const int c_lo = lo - (kbase + j * BNK);
        const int c_hi = t - (kbase + j * BNK);
        uint32_t r0[32], r1[32];
        tmem_ld32(tsrc, r0);
        tmem_ld32(tsrc + 32, r1);
        tmem_ld_wait();
        // whole tile visible to every row of this warp: no per-element mask
        const bool full = __all_sync(0xffffffffu, c_lo <= 0 && c_hi >= BNK);
        float mx = -INFINITY;
        if (full) {
#pragma unroll
          for (int q = 0; q < 32; ++q) mx = fmaxf(mx, fmaxf(__uint_as_float(r0[q]), __uint_as_float(r1[q])));
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            if (q >= c_lo && q < c_hi) mx = fmaxf(mx, __uint_as_float(r0[q]));
            if (q + 32 >= c_lo && q + 32 < c_hi) mx = fmaxf(mx, __uint_as_float(r1[q]));
          }
        }
        mx *= sc;
        // move the reference max only when it grows by more than 2^8
        const bool move = mx > m + kRescaleLog2;
        const float m_new = move ? mx : m;
        const float alpha = (move && m != -INFINITY) ? fast_exp2(m - m_new) : 1.f;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const uint64_t nm2 = f2_pack(-m_use, -m_use);
        // P(i) goes over the S(i) columns: the PV MMA of tile i-2, the last
        // reader of this buffer, was issued before S(i) (whose completion
        // this thread has seen), so it is done
        uint64_t ps2 = f2_pack(0.f, 0.f);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t pk[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int c = cc * 32 + 2 * q;
            const float s0 = __uint_as_float(cc ? r1[2 * q] : r0[2 * q]);
            const float s1 = __uint_as_float(cc ? r1[2 * q + 1] : r0[2 * q + 1]);
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(s0, s1), sc2, nm2), x0, x1);
            float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
            if (!full) {
              p0 = (c >= c_lo && c < c_hi) ? p0 : 0.f;
              p1 = (c + 1 >= c_lo && c + 1 < c_hi) ? p1 : 0.f;
            }
            ps2 = f2_add(ps2, f2_pack(p0, p1));
            pk[q] = pack_bf16(p0, p1);
          }
          tmem_st16(tsrc + cc * 16, pk);
        }
        float psa, psb;
        f2_unpack(ps2, psa, psb);
        l = l * alpha + (psa + psb);
        m = m_new;
        // rare: rescale O, after PV(i-1) has completed
        if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bars[PP_O + 2 * grp + ((i - 1) & 1)], ((i - 1) >> 1) & 1, abort,
                                                 &g_fault_word));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < HD / 32; ++cc) {
            uint32_t r[32];
            tmem_ld32(tO + lane_off + cc * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 32; ++q) r[q] = __float_as_uint(__uint_as_float(r[q]) * alpha);
            tmem_st32(tO + lane_off + cc * 32, r);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars[PP_P + 2 * grp + (i & 1)]);
        if (row == 0) LLATTN_TRACE_K(1, 16 + grp * 24 + i);
      }
      if (!ok) raise_fault(g, kFaultSoftmax, abort);
      if (ok && fuse && L::X_OVER_Q) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[PP_SD], 0, abort, &g_fault_word));
        if (ok) write_lat_rows();
      }
      if (ok && n_mine > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[PP_O + 2 * grp + ((n_mine - 1) & 1)], ((n_mine - 1) >> 1) & 1,
                                               abort, &g_fault_word));
      if (ok && fuse) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[PP_R + grp], 0, abort, &g_fault_word));
        // the per-column constants written by group A
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars[PP_LW + 0], 0, abort, &g_fault_word));
      }
      if (row == 0) LLATTN_TRACE_K(1, 52 + 2 * grp);
      if (!ok) {
        raise_fault(g, kFaultEpilogue, abort);
      } else {
        tc_fence_after();
        const int nk_here = n_mine;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        bf16* dst = local_out + ((int64_t)b * g.T + (valid ? t : 0)) * g.d + (int64_t)h * g.hd;
        if (fuse) {
          // pass 1 over TMEM: gate logits of local = bf16(O / l) and
          // remote = R + b; pass 2: local (over this group's Q tile) and
          // mixed = w local + (1 - w) remote (over its remote operands), then
          // both 128-row tiles to global by TMA (3-D maps clip rows past T)
          uint8_t* ltile = PAIR ? smem + (grp ? L::QB : L::QA) : smem + L::K;
          uint8_t* mtile = PAIR ? xreg : smem + L::V;
          auto tile_chunk = [&](uint8_t* tile, int c) -> uint4* {  // 16-byte chunk c of this row, SW128
            return reinterpret_cast<uint4*>(tile + (c >> 3) * (BM * 128) + row * 128 + (((c & 7) ^ (row & 7)) * 16));
          };
          const float4* b4 = reinterpret_cast<const float4*>(cst);
          const float4* gl4 = reinterpret_cast<const float4*>(cst + HD);
          const float4* gr4 = reinterpret_cast<const float4*>(cst + 2 * HD);
          auto load_row = [&](int cc, float (&lv)[32], float (&rv)[32]) {
            uint32_t ro[32], rr[32];
            if (nk_here > 0) tmem_ld32(tO + lane_off + cc * 32, ro);
            tmem_ld32(tR + lane_off + cc * 32, rr);
            tmem_ld_wait();
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
              const float4 bb = b4[cc * 8 + i4];
              const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int q = 4 * i4 + k;
                lv[q] = nk_here > 0 ? __bfloat162float(__float2bfloat16_rn(__uint_as_float(ro[q]) * inv)) : 0.f;
                rv[q] = __uint_as_float(rr[q]) + bv[k];
              }
            }
          };
          float sl = 0.f, sr = 0.f;
#pragma unroll 1
          for (int cc = 0; cc < HD / 32; ++cc) {
            float lv[32], rv[32];
            load_row(cc, lv, rv);
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
              const float4 ga = gl4[cc * 8 + i4], gb = gr4[cc * 8 + i4];
              sl = fmaf(lv[4 * i4], ga.x, fmaf(lv[4 * i4 + 1], ga.y, fmaf(lv[4 * i4 + 2], ga.z, fmaf(lv[4 * i4 + 3], ga.w, sl))));
              sr = fmaf(rv[4 * i4], gb.x, fmaf(rv[4 * i4 + 1], gb.y, fmaf(rv[4 * i4 + 2], gb.z, fmaf(rv[4 * i4 + 3], gb.w, sr))));
            }
          }
          if (row == 0) LLATTN_TRACE_K(1, 56 + grp);
          const float x = sl + g.gate_bias - sr;
          const float wl = 1.f / (1.f + expf(-x));
          const float wr = 1.f / (1.f + expf(x));
#pragma unroll 1
          for (int cc = 0; cc < HD / 32; ++cc) {
            float lv[32], rv[32];
            load_row(cc, lv, rv);
            uint32_t pl[16], pm[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              pl[q] = pack_bf16(lv[2 * q], lv[2 * q + 1]);
              pm[q] = pack_bf16(wl * lv[2 * q] + wr * rv[2 * q], wl * lv[2 * q + 1] + wr * rv[2 * q + 1]);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              *tile_chunk(ltile, cc * 4 + q) = make_uint4(pl[4 * q], pl[4 * q + 1], pl[4 * q + 2], pl[4 * q + 3]);
              *tile_chunk(mtile, cc * 4 + q) = make_uint4(pm[4 * q], pm[4 * q + 1], pm[4 * q + 2], pm[4 * q + 3]);
            }
          }
          fence_async_smem();
          if (row == 0) LLATTN_TRACE_K(1, 58 + grp);
          mbar_arrive(&bars[PP_EP + grp]);
          if (row == 0) {
            if (mbar_wait(&bars[PP_EP + grp], 0, abort, &g_fault_word)) {
#pragma unroll
              for (int p = 0; p < HD / 64; ++p) {
                tma_store_4d(&tm_lo, ltile + p * (BM * 128), p * 64, h, q0 + grp * BM, b);
                tma_store_4d(&tm_mx, mtile + p * (BM * 128), p * 64, h, q0 + grp * BM, b);
              }
              tma_store_commit();
              LLATTN_TRACE_K(1, 62 + grp);
              tma_store_wait_read();
            } else {
              raise_fault(g, kFaultEpilogue, abort);
            }
          }
        } else {
#pragma unroll 1
          for (int cc = 0; cc < HD / 32; ++cc) {
            uint32_t r[32];
            if (nk_here > 0) {
              tmem_ld32(tO + lane_off + cc * 32, r);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int q = 0; q < 32; ++q) r[q] = 0u;
            }
            uint32_t pk[16];
#pragma unroll
            for (int q = 0; q < 16; ++q)
              pk[q] = pack_bf16(__uint_as_float(r[2 * q]) * inv, __uint_as_float(r[2 * q + 1]) * inv);
            if (valid) {
#pragma unroll
              for (int q = 0; q < 4; ++q)
                if (cc * 32 + q * 8 < g.hd)  // padded head_dim: columns past hd are not stored
                  *reinterpret_cast<uint4*>(dst + cc * 32 + q * 8) =
                      make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
            }
          }
        }
        if (valid) lse_out[((int64_t)b * g.H + h) * g.T + t] = l > 0.f ? (m + log2f(l)) * kLn2 : INFINITY;
      }
      if (row == 0) LLATTN_TRACE_K(1, 53 + 2 * grp);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) LLATTN_TRACE_K(1, 60);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}
