// General bf16 GEMM on the tensor cores (included by local_sm100.cu): the
// remote projection and its gradients when the latent width is not the 64
// columns the fused epilogues hold (the reference's training presets use
// latent_d_model 384 and 512, train.py:71-92):
//   remote  = lat W_rout^T + b_rout          (forward, and recomputed in the backward)
//   dlat    = dR W_rout                      (dR = gradient of remote)
//   dW_rout = dR^T lat,  db_rout = colsum dR (split over rows)
//
// C[M, N] = A[M, K] B[N, K]^T with fp32 accumulation in TMEM. Each operand is
// K-major (rows of K contiguous elements) or MN-major (stored [K, M] with M
// contiguous), read by TMA as 128-byte-swizzled tiles: a K-major tile is 128
// rows x 64 K (one 16 KB copy), an MN-major tile two 64-wide panels of 64 K
// rows (two 8 KB copies). Out-of-range rows / columns / K are zero-filled by
// the copies and masked in the epilogue, so no size needs padding. One
// 128 x 128 output tile per CTA, three-stage ring, two CTAs per SM; warp 0
// loads, warp 1 issues the MMAs, warps 2-5 read the accumulator (thread = row)
// and store it with the optional bias, in bf16 or fp32, through a row map
// (row m -> (m / rows_per_group) * group_stride + (m % rows_per_group) *
// row_step) that lets the forward write remote rows straight into the rows
// of `mixed` the gate kernel reads them from. Optional: column sums of A over
// K (one more MMA per K step against a tile of ones), for db_rout.

struct GemmArgs {
  int M, N, K;
  int a_mn, b_mn;        // 0: K-major, 1: MN-major
  int k_per_split;       // multiple of 64; blockIdx.z = split
  const float* bias;     // [N] or nullptr
  void* C;
  int64_t ldc;           // elements between output rows
  int c_bf16;            // 1: bf16 output, 0: fp32
  int64_t c_split;       // elements between the splits' outputs
  int rows_per_group, group_stride, row_step;
  float* colsum;         // [splits][M] fp32 or nullptr: sum_k A[m, k]
  int64_t colsum_split;  // elements between the splits' column sums
};

struct GemmLayout {
  static constexpr int ST = 3;
  static constexpr int TILE = 128 * 64 * 2;  // 16 KB
  static constexpr int A = 0;
  static constexpr int B = A + ST * TILE;
  static constexpr int ONES = B + ST * TILE;  // 16 x 64 bf16 ones
  static constexpr int BAR = ONES + 2048;
  static constexpr int BYTES = BAR + 128;
  static_assert(BYTES + 1024 <= 113 * 1024, "two CTAs per SM");
};

enum { GM_F = 0, GM_E = 3, GM_DONE = 6, GM_NB = 7 };

__global__ void __launch_bounds__(192, 2)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, Geom g,
                   GemmArgs p) {
  using L = GemmLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + GM_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n0 = blockIdx.x * 128, m0 = blockIdx.y * 128, split = blockIdx.z;
  const int ka = split * p.k_per_split, kb = min(p.K, ka + p.k_per_split);
  const int nk = kb > ka ? cdiv(kb - ka, 64) : 0;
  const bool want_colsum = p.colsum != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::ST; ++s) {
      mbar_init(&bars[GM_F + s], 1);
      mbar_init(&bars[GM_E + s], 1);
    }
    mbar_init(&bars[GM_DONE], 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (want_colsum) {  // ones tile, K-major swizzled (all elements equal: the swizzle is moot)
    uint4* o = reinterpret_cast<uint4*>(smem + L::ONES);
    for (int i = threadIdx.x; i < 2048 / 16; i += blockDim.x)
      o[i] = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    fence_async_smem();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // C tile at [0, 128), column sums at [128, 144)

  if (warp == 0) {
    if (lane == 0 && nk > 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_b);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % L::ST, k0 = ka + i * 64;
        if (i >= L::ST && !mbar_wait(&bars[GM_E + s], ((i / L::ST) - 1) & 1, abort, &g_fault_word)) {
          raise_fault(g, kFaultProducer, abort);
          break;
        }
        mbar_expect_tx(&bars[GM_F + s], 2 * L::TILE);
        uint8_t* sa = smem + L::A + s * L::TILE;
        uint8_t* sb = smem + L::B + s * L::TILE;
        if (p.a_mn) {
          tma_load_2d(&tm_a, &bars[GM_F + s], sa, m0, k0);
          tma_load_2d(&tm_a, &bars[GM_F + s], sa + L::TILE / 2, m0 + 64, k0);
        } else {
          tma_load_2d(&tm_a, &bars[GM_F + s], sa, k0, m0);
        }
        if (p.b_mn) {
          tma_load_2d(&tm_b, &bars[GM_F + s], sb, n0, k0);
          tma_load_2d(&tm_b, &bars[GM_F + s], sb + L::TILE / 2, n0 + 64, k0);
        } else {
          tma_load_2d(&tm_b, &bars[GM_F + s], sb, k0, n0);
        }
        issued = i + 1;
      }
      if (*abort) {  // let the copies already issued land before the CTA can exit
        volatile int none = 0;
        volatile unsigned gnone = 0;
        for (int i = issued - L::ST < 0 ? 0 : issued - L::ST; i < issued; ++i)
          mbar_wait(&bars[GM_F + i % L::ST], (i / L::ST) & 1, &none, &gnone, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nk > 0) {
      const uint32_t id = idesc_bf16_f32(128, 128, p.a_mn != 0, p.b_mn != 0);
      const uint32_t id1 = idesc_bf16_f32(128, 16, p.a_mn != 0, false);
      const uint64_t d1 = desc_sw128(smem_u32(smem + L::ONES), 16, 1024);
      // K-major: K step of 16 = 32 bytes within the 128-byte rows; MN-major:
      // 16 rows of 128 bytes, panels of 64 M (N) at 8 KB
      const uint32_t a_step = p.a_mn ? 2048 : 32, b_step = p.b_mn ? 2048 : 32;
      const uint32_t a_lbo = p.a_mn ? L::TILE / 2 : 16, b_lbo = p.b_mn ? L::TILE / 2 : 16;
      bool ok = true;
      for (int i = 0; ok && i < nk; ++i) {
        const int s = i % L::ST;
        if (!(ok = mbar_wait(&bars[GM_F + s], (i / L::ST) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint64_t da = desc_sw128(smem_u32(smem + L::A + s * L::TILE), a_lbo, 1024);
        const uint64_t db = desc_sw128(smem_u32(smem + L::B + s * L::TILE), b_lbo, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          mma_bf16(tmem, desc_add(da, kk * a_step), desc_add(db, kk * b_step), id, acc);
          if (want_colsum) mma_bf16(tmem + 128, desc_add(da, kk * a_step), desc_add(d1, kk * 32), id1, acc);
        }
        mma_commit(&bars[GM_E + s]);
      }
      mma_commit(&bars[GM_DONE]);
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    bool ok = true;
    if (nk > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars[GM_DONE], 0, abort, &g_fault_word));
    if (!ok) {
      raise_fault(g, kFaultEpilogue, abort);
    } else {
      tc_fence_after();
      const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
      const int m = m0 + 32 * (warp & 3) + lane;  // TMEM lane = output row
      const bool row_ok = m < p.M;
      const int64_t orow = row_ok ? (int64_t)(m / p.rows_per_group) * p.group_stride +
                                        (int64_t)(m % p.rows_per_group) * p.row_step
                                  : 0;
      const bool vec = (p.ldc % 8) == 0;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const int nc = n0 + cc * 32;
        if (nc >= p.N) break;  // warp-uniform
        uint32_t r[32];
        if (nk > 0) {
          tmem_ld32(tmem + lane_off + cc * 32, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) r[q] = 0u;
        }
        if (!row_ok) continue;
        float v[32];
        const bool full = nc + 32 <= p.N && vec;
        if (p.bias && full && ((reinterpret_cast<uintptr_t>(p.bias + nc) & 15) == 0)) {
          const float4* b4 = reinterpret_cast<const float4*>(p.bias + nc);  // 8 vector loads, not 32
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = __ldg(b4 + q);
            v[4 * q] = __uint_as_float(r[4 * q]) + bb.x;
            v[4 * q + 1] = __uint_as_float(r[4 * q + 1]) + bb.y;
            v[4 * q + 2] = __uint_as_float(r[4 * q + 2]) + bb.z;
            v[4 * q + 3] = __uint_as_float(r[4 * q + 3]) + bb.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            const int n = nc + q;
            v[q] = __uint_as_float(r[q]) + ((p.bias && n < p.N) ? __ldg(p.bias + n) : 0.f);
          }
        }
        if (p.c_bf16) {
          bf16* dst = static_cast<bf16*>(p.C) + (int64_t)split * p.c_split + orow * p.ldc + nc;
          if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              reinterpret_cast<uint4*>(dst)[q] =
                  make_uint4(pack_bf16(v[8 * q], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                             pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7]));
          } else {
            for (int q = 0; q < 32 && nc + q < p.N; ++q) dst[q] = __float2bfloat16_rn(v[q]);
          }
        } else {
          float* dst = static_cast<float*>(p.C) + (int64_t)split * p.c_split + orow * p.ldc + nc;
          if (full && (p.ldc % 4) == 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          } else {
            for (int q = 0; q < 32 && nc + q < p.N; ++q) dst[q] = v[q];
          }
        }
      }
      if (want_colsum && blockIdx.x == 0) {  // the column sums do not depend on the N tile
        uint32_t r1[16];
        if (nk > 0) {
          tmem_ld16(tmem + lane_off + 128, r1);
          tmem_ld_wait();
        } else {
          r1[0] = 0u;
        }
        if (row_ok) p.colsum[(int64_t)split * p.colsum_split + m] = __uint_as_float(r1[0]);
      }
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

// Persistent variant (no column sums): one CTA per SM slot walks the output
// tiles t = blockIdx.x + k * gridDim.x (N tiles fastest, so the CTAs running
// together share A rows in L2). The shared-memory ring continues across
// tiles, so the next tile's loads start while this tile's MMAs run, and the
// accumulator is double-buffered in TMEM (two 128-column buffers): the
// epilogue of tile k reads one buffer while the MMAs of tile k+1 fill the
// other. Barriers: ring full / empty per stage, accumulator full / empty per
// buffer.
enum { GP_F = 0, GP_E = 3, GP_AF = 6, GP_AE = 8, GP_NB = 10 };

__global__ void __launch_bounds__(192, 2)
    gemm_tc_persistent_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                              Geom g, GemmArgs p) {
  using L = GemmLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + GP_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_nt = cdiv(p.N, 128), n_tiles = n_nt * cdiv(p.M, 128);
  const int nk = cdiv(p.K, 64);

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::ST; ++s) {
      mbar_init(&bars[GP_F + s], 1);
      mbar_init(&bars[GP_E + s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars[GP_AF + b], 1);
      mbar_init(&bars[GP_AE + b], 128);
    }
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
  const uint32_t tmem = *tmem_slot;  // accumulator buffer b at [128 b, 128 b + 128)

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_b);
      int it = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
        const int n0 = (t % n_nt) * 128, m0 = (t / n_nt) * 128;
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % L::ST, k0 = i * 64;
          if (it >= L::ST && !(ok = mbar_wait(&bars[GP_E + s], ((it / L::ST) - 1) & 1, abort, &g_fault_word)))
            break;
          mbar_expect_tx(&bars[GP_F + s], 2 * L::TILE);
          uint8_t* sa = smem + L::A + s * L::TILE;
          uint8_t* sb = smem + L::B + s * L::TILE;
          if (p.a_mn) {
            tma_load_2d(&tm_a, &bars[GP_F + s], sa, m0, k0);
            tma_load_2d(&tm_a, &bars[GP_F + s], sa + L::TILE / 2, m0 + 64, k0);
          } else {
            tma_load_2d(&tm_a, &bars[GP_F + s], sa, k0, m0);
          }
          if (p.b_mn) {
            tma_load_2d(&tm_b, &bars[GP_F + s], sb, n0, k0);
            tma_load_2d(&tm_b, &bars[GP_F + s], sb + L::TILE / 2, n0 + 64, k0);
          } else {
            tma_load_2d(&tm_b, &bars[GP_F + s], sb, k0, n0);
          }
          issued = it + 1;
        }
      }
      if (!ok) {
        raise_fault(g, kFaultProducer, abort);
        volatile int none = 0;  // let the copies already issued land before the CTA can exit
        volatile unsigned gnone = 0;
        for (int i = issued - L::ST < 0 ? 0 : issued - L::ST; i < issued; ++i)
          mbar_wait(&bars[GP_F + i % L::ST], (i / L::ST) & 1, &none, &gnone, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id = idesc_bf16_f32(128, 128, p.a_mn != 0, p.b_mn != 0);
      const uint32_t a_step = p.a_mn ? 2048 : 32, b_step = p.b_mn ? 2048 : 32;
      const uint32_t a_lbo = p.a_mn ? L::TILE / 2 : 16, b_lbo = p.b_mn ? L::TILE / 2 : 16;
      int it = 0, k = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++k) {
        const int buf = k & 1;
        // the epilogue has read this buffer's previous tile (k - 2)
        if (k >= 2 && !(ok = mbar_wait(&bars[GP_AE + buf], ((k >> 1) - 1) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % L::ST;
          if (!(ok = mbar_wait(&bars[GP_F + s], (it / L::ST) & 1, abort, &g_fault_word))) break;
          tc_fence_after();
          const uint64_t da = desc_sw128(smem_u32(smem + L::A + s * L::TILE), a_lbo, 1024);
          const uint64_t db = desc_sw128(smem_u32(smem + L::B + s * L::TILE), b_lbo, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem + 128 * buf, desc_add(da, kk * a_step), desc_add(db, kk * b_step), id,
                     (i > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&bars[GP_E + s]);
        }
        if (!ok) break;
        mma_commit(&bars[GP_AF + buf]);
      }
      if (!ok) raise_fault(g, kFaultMma, abort);
    }
  } else {
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const bool vec = (p.ldc % 8) == 0;
    int k = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++k) {
      const int buf = k & 1, n0 = (t % n_nt) * 128, m0 = (t / n_nt) * 128;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[GP_AF + buf], (k >> 1) & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      const int m = m0 + 32 * (warp & 3) + lane;
      const bool row_ok = m < p.M;
      const int64_t orow = row_ok ? (int64_t)(m / p.rows_per_group) * p.group_stride +
                                        (int64_t)(m % p.rows_per_group) * p.row_step
                                  : 0;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const int nc = n0 + cc * 32;
        if (nc >= p.N) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld32(tmem + 128 * buf + lane_off + cc * 32, r);
        tmem_ld_wait();
        if (!row_ok) continue;
        float v[32];
        const bool full = nc + 32 <= p.N && vec;
        if (p.bias && full && ((reinterpret_cast<uintptr_t>(p.bias + nc) & 15) == 0)) {
          const float4* b4 = reinterpret_cast<const float4*>(p.bias + nc);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = __ldg(b4 + q);
            v[4 * q] = __uint_as_float(r[4 * q]) + bb.x;
            v[4 * q + 1] = __uint_as_float(r[4 * q + 1]) + bb.y;
            v[4 * q + 2] = __uint_as_float(r[4 * q + 2]) + bb.z;
            v[4 * q + 3] = __uint_as_float(r[4 * q + 3]) + bb.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            const int n = nc + q;
            v[q] = __uint_as_float(r[q]) + ((p.bias && n < p.N) ? __ldg(p.bias + n) : 0.f);
          }
        }
        if (p.c_bf16) {
          bf16* dst = static_cast<bf16*>(p.C) + orow * p.ldc + nc;
          if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              reinterpret_cast<uint4*>(dst)[q] =
                  make_uint4(pack_bf16(v[8 * q], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                             pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7]));
          } else {
            for (int q = 0; q < 32 && nc + q < p.N; ++q) dst[q] = __float2bfloat16_rn(v[q]);
          }
        } else {
          float* dst = static_cast<float*>(p.C) + orow * p.ldc + nc;
          if (full && (p.ldc % 4) == 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          } else {
            for (int q = 0; q < 32 && nc + q < p.N; ++q) dst[q] = v[q];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[GP_AE + buf]);  // this buffer may take the tile after next
    }
    if (!ok) raise_fault(g, kFaultEpilogue, abort);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}
