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

template <int HD>
struct GbLayout {
  static constexpr int LAT = 0;                    // 128 x 64 bf16
  static constexpr int W = LAT + BM * 128;         // 2 x (HD x 64 bf16)
  static constexpr int DR = W + 2 * HD * 128;      // 2 x (128 x HD bf16)
  static constexpr int RED = DR + 2 * BM * HD * 2; // 4 warps x 2 x HD floats
  static constexpr int BAR = RED + 4 * 2 * HD * 4;
  static constexpr int BYTES = BAR + 256;
};

enum { GB_W = 0, GB_R = 2, GB_DR = 4, GB_DL = 6, GB_NB = 8 };

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

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(p[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

template <int HD>
__global__ void __launch_bounds__(192, 1)
    gate_bwd_tc_kernel(Geom g, const bf16* __restrict__ local_out, const bf16* __restrict__ lat,
                       const bf16* __restrict__ w_rout, const float* __restrict__ b_rout,
                       const float* __restrict__ gl, const float* __restrict__ gr, const bf16* __restrict__ dmixed,
                       bf16* __restrict__ dl, float* __restrict__ delta, bf16* __restrict__ dr,
                       float* __restrict__ dlat_tok, float* __restrict__ dg_part) {
  using L = GbLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + GB_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = blockIdx.y, t0 = blockIdx.x * BM;
  const int H = g.H;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[GB_W + s], BM);
      mbar_init(&bars[GB_R + s], 1);
      mbar_init(&bars[GB_DR + s], BM);
      mbar_init(&bars[GB_DL + s], 1);
    }
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
  const uint32_t tmem = *tmem_slot;  // R_h buffers at [0,HD) and [HD,2HD); dlat at 256
  const uint32_t tDL = tmem + 256;
  float* red = reinterpret_cast<float*>(smem + L::RED);

  if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idR = idesc_bf16_f32(BM, HD, false, false);  // lat . W_h^T
      constexpr uint32_t idL = idesc_bf16_f32(BM, 64, false, true);   // dR_h . W_h
      const uint32_t la = smem_u32(smem + L::LAT);
      bool ok = true;
      auto issue_r = [&](int h) -> bool {
        const int s = h & 1;
        if (!mbar_wait(&bars[GB_W + s], (h >> 1) & 1, abort, &g_fault_word)) return false;
        tc_fence_after();
        const uint32_t wa = smem_u32(smem + L::W + s * HD * 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(tmem + s * HD, desc_sw128(la + kk * 32, 16, 1024), desc_sw128(wa + kk * 32, 16, 1024), idR,
                   kk > 0);
        mma_commit(&bars[GB_R + s]);
        return true;
      };
      ok = issue_r(0);
      for (int h = 0; ok && h < H; ++h) {
        if (h + 1 < H && !(ok = issue_r(h + 1))) break;
        const int s = h & 1;
        if (!(ok = mbar_wait(&bars[GB_DR + s], (h >> 1) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint32_t da = smem_u32(smem + L::DR + s * BM * HD * 2);
        const uint32_t wa = smem_u32(smem + L::W + s * HD * 128);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_bf16(tDL, desc_sw128(da + (kk / 4) * (BM * 128) + (kk % 4) * 32, 16, 1024),
                   desc_sw128(wa + kk * 2048, 0, 1024), idL, (h > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars[GB_DL + s]);
      }
      if (!ok) raise_fault(kFaultMma, abort);
    }
  } else if (warp >= 2) {
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const int t = t0 + row;
    const bool valid = t < g.T;
    const int64_t tok = (int64_t)b * g.T + (valid ? t : 0);
    // lat row of this token, 128-byte swizzled rows
    {
      const uint4* src = reinterpret_cast<const uint4*>(lat + ((int64_t)b * g.Tq + (valid ? t / g.qbs : 0)) * 64);
      uint8_t* d = smem + L::LAT + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(d + ((c ^ (row & 7)) * 16)) = src[c];
    }
    auto write_w = [&](int h) {
      if (row < HD) {
        const uint4* src = reinterpret_cast<const uint4*>(w_rout + ((int64_t)h * HD + row) * 64);
        uint8_t* d = smem + L::W + (h & 1) * HD * 128 + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(d + ((c ^ (row & 7)) * 16)) = src[c];
      }
      fence_async_smem();
      mbar_arrive(&bars[GB_W + (h & 1)]);
    };
    write_w(0);
    // per-warp dg accumulators in shared memory; lane owns column cc*32+lane
    float* wred = red + (warp & 3) * 2 * HD;
    for (int e = lane; e < 2 * HD; e += 32) wred[e] = 0.f;
    bool ok = true;
    for (int h = 0; h < H; ++h) {
      const int s = h & 1;
      if (h >= 1) {  // dlat MMA of head h-1 done: W[(h+1)&1] and DR[s] are free
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_DL + ((h - 1) & 1)], ((h - 1) >> 1) & 1, abort,
                                               &g_fault_word));
        if (!ok) break;
      }
      if (h + 1 < H) write_w(h + 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_R + s], (h >> 1) & 1, abort, &g_fault_word));
      if (!ok) break;
      tc_fence_after();
      const bf16* lrow = local_out + tok * g.d + (int64_t)h * HD;
      const bf16* mrow = dmixed + tok * g.d + (int64_t)h * HD;
      const float* bh = b_rout + (int64_t)h * HD;
      // pass 1: gate logits and dw
      float sl = 0.f, sr = 0.f, dw = 0.f;
#pragma unroll
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_off + s * HD + cc * 32, rr);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float lv[8], mv[8];
          unpack8(reinterpret_cast<const uint4*>(lrow + cc * 32)[q], lv);
          unpack8(reinterpret_cast<const uint4*>(mrow + cc * 32)[q], mv);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int c = cc * 32 + q * 8 + i;
            const float rv = __uint_as_float(rr[q * 8 + i]) + __ldg(bh + c);
            sl = fmaf(lv[i], __ldg(gl + c), sl);
            sr = fmaf(rv, __ldg(gr + c), sr);
            dw = fmaf(mv[i], lv[i] - rv, dw);
          }
        }
      }
      const float x = sl + g.gate_bias - sr;
      const float w = 1.f / (1.f + expf(-x));
      const float wr = 1.f / (1.f + expf(x));
      const float ds = valid ? dw * w * wr : 0.f;
      // pass 2: dL, D, dR, dg
      float dsum = 0.f;
      uint8_t* drow_s = smem + L::DR + s * BM * HD * 2 + row * 128;
#pragma unroll 1
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_off + s * HD + cc * 32, rr);
        tmem_ld_wait();
        float al[32];
        uint32_t pdl[16], pdr[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float lv[8], mv[8];
          unpack8(reinterpret_cast<const uint4*>(lrow + cc * 32)[q], lv);
          unpack8(reinterpret_cast<const uint4*>(mrow + cc * 32)[q], mv);
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            float dlv[2], drv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int c = cc * 32 + q * 8 + i + u;
              const float rv = __uint_as_float(rr[q * 8 + i + u]) + __ldg(bh + c);
              const float a = __bfloat162float(__float2bfloat16_rn(w * mv[i + u] + ds * __ldg(gl + c)));
              dlv[u] = a;
              dsum = fmaf(a, lv[i + u], dsum);
              drv[u] = wr * mv[i + u] - ds * __ldg(gr + c);
              al[q * 8 + i + u] = ds * lv[i + u];
            }
            pdl[(q * 8 + i) / 2] = pack_bf16(dlv[0], dlv[1]);
            pdr[(q * 8 + i) / 2] = pack_bf16(drv[0], drv[1]);
          }
        }
        if (valid) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 vl = make_uint4(pdl[4 * q], pdl[4 * q + 1], pdl[4 * q + 2], pdl[4 * q + 3]);
            const uint4 vr = make_uint4(pdr[4 * q], pdr[4 * q + 1], pdr[4 * q + 2], pdr[4 * q + 3]);
            reinterpret_cast<uint4*>(dl + tok * g.d + (int64_t)h * HD + cc * 32)[q] = vl;
            reinterpret_cast<uint4*>(dr + tok * g.d + (int64_t)h * HD + cc * 32)[q] = vr;
          }
        }
        // dR row into the swizzled A tile (rows past T hold zeros)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = cc * 4 + q;  // 16-byte chunk along HD
          const uint4 vr = valid ? make_uint4(pdr[4 * q], pdr[4 * q + 1], pdr[4 * q + 2], pdr[4 * q + 3])
                                 : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(drow_s + (chunk >> 3) * (BM * 128) + ((chunk & 7) ^ (row & 7)) * 16) = vr;
        }
        wred[cc * 32 + lane] += butterfly32(al, lane);
        {
          float ar[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) ar[i] = -ds * (__uint_as_float(rr[i]) + __ldg(bh + cc * 32 + i));
          wred[HD + cc * 32 + lane] += butterfly32(ar, lane);
        }
      }
      if (valid) delta[((int64_t)b * H + h) * g.T + t] = dsum;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[GB_DR + s]);
    }
    if (!ok) raise_fault(kFaultSoftmax, abort);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars[GB_DL + ((H - 1) & 1)], ((H - 1) >> 1) & 1, abort,
                                                   &g_fault_word));
    if (!ok) {
      raise_fault(kFaultEpilogue, abort);
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
            d[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                               __uint_as_float(r[4 * q + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // partial [cta][2*HD] (dg_l half, dg_r half) summed over the compute warps
  for (int e = threadIdx.x; e < 2 * HD; e += 192) {
    const float v = red[e] + red[2 * HD + e] + red[4 * HD + e] + red[6 * HD + e];
    dg_part[((int64_t)b * gridDim.x + blockIdx.x) * 2 * HD + e] = v;
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------

constexpr int DW_ST = 4;  // pipeline stages of 64 tokens

struct DwLayout {
  static constexpr int A = 0;                    // DW_ST x (64 tokens x 128 cols bf16) = 16 KB each
  static constexpr int B = A + DW_ST * 16384;    // DW_ST x (64 tokens x 64 bf16) = 8 KB each
  static constexpr int BAR = B + DW_ST * 8192;
  static constexpr int BYTES = BAR + 256;
};

enum { DW_FA = 0, DW_FB = DW_ST, DW_E = 2 * DW_ST, DW_DONE = 3 * DW_ST, DW_NB = 3 * DW_ST + 1 };

__global__ void __launch_bounds__(192, 1)
    rout_dw_tc_kernel(const __grid_constant__ CUtensorMap tm_dr, Geom g, const bf16* __restrict__ lat,
                      float* __restrict__ dw_part, float* __restrict__ db_part, int n_split) {
  using L = DwLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + DW_NB);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c0 = blockIdx.x * 128, split = blockIdx.y;
  const int n_tok = g.B * g.T;
  const int per = cdiv(cdiv(n_tok, n_split), 64) * 64;
  const int na = split * per, nb = min(n_tok, na + per);
  const int nch = nb > na ? cdiv(nb - na, 64) : 0;

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
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nch > 0) {
      prefetch_tmap(&tm_dr);
      int issued = 0;
      for (int i = 0; i < nch; ++i) {
        const int s = i % DW_ST;
        if (i >= DW_ST && !mbar_wait(&bars[DW_E + s], ((i / DW_ST) - 1) & 1, abort, &g_fault_word)) {
          raise_fault(kFaultProducer, abort);
          break;
        }
        mbar_expect_tx(&bars[DW_FA + s], 16384);
        // rows past this split's range belong to the next split: they are
        // loaded but zeroed out of the B tile, so they contribute nothing
        tma_load_2d(&tm_dr, &bars[DW_FA + s], smem + L::A + s * 16384, c0, na + i * 64);
        tma_load_2d(&tm_dr, &bars[DW_FA + s], smem + L::A + s * 16384 + 8192, c0 + 64, na + i * 64);
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
      bool ok = true;
      for (int i = 0; ok && i < nch; ++i) {
        const int s = i % DW_ST;
        if (!(ok = mbar_wait(&bars[DW_FA + s], (i / DW_ST) & 1, abort, &g_fault_word))) break;
        if (!(ok = mbar_wait(&bars[DW_FB + s], (i / DW_ST) & 1, abort, &g_fault_word))) break;
        tc_fence_after();
        const uint32_t aa = smem_u32(smem + L::A + s * 16384), ba = smem_u32(smem + L::B + s * 8192);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(tmem, desc_sw128(aa + kk * 2048, 8192, 1024), desc_sw128(ba + kk * 2048, 0, 1024), id,
                   (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars[DW_E + s]);
      }
      mma_commit(&bars[DW_DONE]);
      if (!ok) raise_fault(kFaultMma, abort);
    }
  } else {
    const int tid = threadIdx.x - 64;  // 0..127: column c0 + tid, and B-tile writer
    float db = 0.f;
    bool ok = true;
    for (int i = 0; i < nch; ++i) {
      const int s = i % DW_ST;
      if (i >= DW_ST) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[DW_E + s], ((i / DW_ST) - 1) & 1, abort, &g_fault_word));
        if (!ok) break;
      }
      // B tile: 64 token rows of lat (row r of token n = b*T + t -> lat row b*Tq + t/qbs)
      {
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
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[DW_FA + s], (i / DW_ST) & 1, abort, &g_fault_word));
      if (!ok) break;
      // db: column sum of the dR tile over its valid rows
      {
        const uint8_t* a = smem + L::A + s * 16384 + (tid >> 6) * 8192;
        const int cc = tid & 63, chunk = cc >> 3, e = cc & 7;
        const int rows = min(64, nb - (na + i * 64));
        for (int r = 0; r < rows; ++r)
          db += __bfloat162float(*reinterpret_cast<const bf16*>(a + r * 128 + ((chunk ^ (r & 7)) * 16) + e * 2));
      }
      fence_async_smem();
      mbar_arrive(&bars[DW_FB + s]);
    }
    if (!ok) raise_fault(kFaultSoftmax, abort);
    const int c = c0 + tid;
    if (ok && nch > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars[DW_DONE], 0, abort, &g_fault_word));
    if (!ok) {
      raise_fault(kFaultEpilogue, abort);
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
      if (c < g.d) db_part[(int64_t)split * g.d + c] = db;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 64);
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
