// Latent branch: causal-chunk attention of latent query rows against the
// pooled chunk keys/values (models.py:361-375), forward and backward.
//
// rq [B,Tq,Lh,ldh], gkv [B,Nc,2,Lh,ldh] (gk = slot 0, gv = slot 1).
// Row r sees chunks j < qid(r); a row with qid = 0 outputs 0 (models.py:366-373).
// The work is tiny next to the local branch (Nc <= 512 keys of ldh <= 64), so
// these kernels use fp32 FMAs with the per-(b, latent head) keys staged in
// shared memory; ldh is padded with zeros up to the template width L.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace llattn {
namespace {


// ---------------------------------------------------------------------------
// Backward. With P = softmax(s) (s = lat_scale * rq.gk), dP = dlat.gv,
// delta = dlat.lat, dS = P (dP - delta):
//   drq = lat_scale * sum_j dS gk_j,  dgk_j = lat_scale * sum_r dS rq_r,
//   dgv_j = sum_r P dlat_r.
// One kernel: a CTA owns (b, latent head, row split) and walks its 64-row
// blocks (interleaved over the splits, so early rows with few visible chunks
// and late rows with many spread evenly). Per row block, pass 1 sums
// delta = sum_j P_j (dlat.gv_j) over the 64-key tiles in fp32 (not from the
// stored, rounded lat: with long chunks the pooled values are nearly equal
// and dS cancels, so delta must be consistent with P to working precision);
// pass 2 forms P and dS per tile in shared memory, accumulates drq in
// registers and adds dgk / dgv into the CTA's own partial slice (plain
// read-modify-write by the owning thread: no atomics). A reduce sums the
// per-split partials in a fixed order, so the result is deterministic.
// S and dP of a 64x64 tile: each thread a 4-row x 4-key block, operands as
// float4 from shared memory (8 FMAs per load); with a single key tile (the
// usual case) pass 2 reuses pass 1's P and dP instead of recomputing them.

constexpr int kLatRows = 64, kLatKeys = 64;
constexpr float kLatLog2e = 1.4426950408889634f;

template <int L>
struct LatBwdSmem {
  static constexpr int LS = L + 4;          // operand row stride (floats; 16-byte rows)
  static constexpr int PS = kLatKeys + 4;   // P / dS row stride
  static constexpr int RQ = 0, DL = RQ + kLatRows * LS, K = DL + kLatRows * LS, V = K + kLatKeys * LS;
  static constexpr int P = V + kLatKeys * LS, DS = P + kLatRows * PS;
  static constexpr int LSE = DS + kLatRows * PS, DELTA = LSE + kLatRows, QID = DELTA + kLatRows;
  static constexpr int FLOATS = QID + kLatRows;
};

// ONE: all chunk keys fit one 64-key tile (Nc <= 64): the keys are staged
// once per CTA and the dgk / dgv accumulators stay in registers across the
// CTA's row blocks (a single store of the partial at the end).
template <typename T, int L, bool ONE>
__global__ void __launch_bounds__(256, 2) latent_bwd_kernel(Geom g, const T* __restrict__ rq,
                                                         const T* __restrict__ gkv,
                                                         const float* __restrict__ lat_lse,
                                                         const float* __restrict__ dlat, T* __restrict__ drq,
                                                         float* __restrict__ part, int n_split, int n_kg,
                                                         float* __restrict__ drq_part) {
  using S = LatBwdSmem<L>;
  constexpr int LS = S::LS, PS = S::PS, EQ = L / 4;
  extern __shared__ float4 smem_lat4[];
  float* sm = reinterpret_cast<float*>(smem_lat4);
  float *s_rq = sm + S::RQ, *s_dl = sm + S::DL, *s_k = sm + S::K, *s_v = sm + S::V;
  float *s_p = sm + S::P, *s_ds = sm + S::DS, *s_lse = sm + S::LSE, *s_delta = sm + S::DELTA;
  int* s_qid = reinterpret_cast<int*>(sm + S::QID);
  // blockIdx.x = row split * n_kg + key group: with n_kg > 1 (several key
  // tiles, too few row splits to fill the GPU) every CTA of a row split sums
  // delta over all keys (pass 1) but forms dS, drq and dgk/dgv only for the
  // key tiles kt = key group (mod n_kg); its drq goes to drq_part[key group]
  // (fp32), summed by a fixed-order reduce.
  const int b = blockIdx.z, lh = blockIdx.y, split = blockIdx.x / n_kg, kgrp = blockIdx.x % n_kg;
  const int tid = threadIdx.x;
  const float sc2 = g.lat_scale * kLatLog2e;
  const int rg = tid >> 4, kg = tid & 15;  // S / dP block: rows 4rg + i, keys kg + 16u
  const int own = tid >> 2, eq = tid & 3;  // drq row / dgk,dgv key, and its e-quarter
  float* my_part = part + ((int64_t)blockIdx.x * g.B + b) * g.Nc * 2 * g.Ld + lh * g.ldh;

  // this CTA's partial slice starts at zero (same thread mapping as the adds)
  if (!ONE)
  for (int j = own; j < g.Nc; j += kLatKeys)
#pragma unroll
    for (int u = 0; u < EQ; ++u) {
      const int e = eq * EQ + u;
      if (e < g.ldh) {
        my_part[(int64_t)(2 * j) * g.Ld + e] = 0.f;
        my_part[(int64_t)(2 * j + 1) * g.Ld + e] = 0.f;
      }
    }

  auto load_keys = [&](int j0) {
    for (int idx = tid; idx < kLatKeys * L; idx += 256) {
      const int jj = idx / L, e = idx % L, j = j0 + jj;
      float kv = 0.f, vv = 0.f;
      if (j < g.Nc && e < g.ldh) {
        const int64_t base = ((int64_t)(b * g.Nc + j) * 2 * g.Lh + lh) * g.ldh + e;
        kv = to_f<T>(gkv[base]);
        vv = to_f<T>(gkv[base + (int64_t)g.Lh * g.ldh]);
      }
      s_k[jj * LS + e] = kv;
      s_v[jj * LS + e] = vv;
    }
  };
  // P and dP of this thread's 4 rows (4rg + i) x 4 keys (kg + 16u) of the
  // tile at j0 into s_p / s_ds; returns nothing, masks keys j >= qid(row).
  // (Keys kg + 16u: the 8 lanes of a quarter warp read 8 distinct 16-byte
  // bank groups of s_k / s_v.)
  auto tile_pdp = [&](int j0) {
    // S block, then dP block (fewer live registers than both at once)
    float sa[4][4], da[4][4];
    auto block = [&](const float* x, const float* y, float (&acc)[4][4]) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[i][u] = 0.f;
#pragma unroll
      for (int e = 0; e < L; e += 4) {
        float4 a[4], k[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i] = *reinterpret_cast<const float4*>(x + (4 * rg + i) * LS + e);
          k[i] = *reinterpret_cast<const float4*>(y + (kg + 16 * i) * LS + e);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            acc[i][u] = fmaf(a[i].x, k[u].x, fmaf(a[i].y, k[u].y, fmaf(a[i].z, k[u].z, fmaf(a[i].w, k[u].w, acc[i][u]))));
      }
    };
    block(s_rq, s_k, sa);
    block(s_dl, s_v, da);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ri = 4 * rg + i;
      const float lse2 = s_lse[ri];
      const int qid = s_qid[ri];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int jj = kg + 16 * u;
        s_p[ri * PS + jj] = j0 + jj < qid ? exp2f(fmaf(sa[i][u], sc2, -lse2)) : 0.f;
        s_ds[ri * PS + jj] = da[i][u];
      }
    }
  };

  // rq / dlat of a row block, loaded into registers one block ahead
  constexpr int NPRE = kLatRows * L / 256;
  float pre_a[NPRE], pre_d[NPRE];
  auto prefetch_rows = [&](int rb) {
#pragma unroll
    for (int k = 0; k < NPRE; ++k) {
      const int idx = tid + 256 * k, i = idx / L, e = idx % L, r = rb * kLatRows + i;
      pre_a[k] = pre_d[k] = 0.f;
      if (r < g.Tq && e < g.ldh) {
        pre_a[k] = to_f<T>(rq[((int64_t)(b * g.Tq + r) * g.Lh + lh) * g.ldh + e]);
        pre_d[k] = dlat[(int64_t)(b * g.Tq + r) * g.Ld + lh * g.ldh + e];
      }
    }
  };
  float ak1[EQ], av1[EQ];  // ONE: dgk / dgv of key `own` over all this CTA's rows
#pragma unroll
  for (int u = 0; u < EQ; ++u) ak1[u] = av1[u] = 0.f;
  if (ONE) load_keys(0);
  const int n_rb = cdiv(g.Tq, kLatRows);
  if (split < n_rb) prefetch_rows(split);
  for (int rb = split; rb < n_rb; rb += n_split) {
    const int r0 = rb * kLatRows;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NPRE; ++k) {
      const int idx = tid + 256 * k, i = idx / L, e = idx % L;
      s_rq[i * LS + e] = pre_a[k];
      s_dl[i * LS + e] = pre_d[k];
    }
    if (rb + n_split < n_rb) prefetch_rows(rb + n_split);
    if (tid < kLatRows) {
      const int r = r0 + tid;
      const bool ok = r < g.Tq;
      s_lse[tid] = ok ? lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r] * kLatLog2e : INFINITY;
      s_qid[tid] = ok ? row_qid(g, r) : 0;
      s_delta[tid] = 0.f;
    }
    const int jmax = row_qid(g, min(r0 + kLatRows - 1, g.Tq - 1));  // keys j < jmax are visible
    const int n_kt = cdiv(jmax, kLatKeys);
    // pass 1: delta = sum_j P dP (P, dP of the last tile stay in s_p / s_ds)
    for (int kt = 0; kt < n_kt; ++kt) {
      __syncthreads();
      if (!ONE) {
        load_keys(kt * kLatKeys);
        __syncthreads();
      }
      tile_pdp(kt * kLatKeys);
      // each thread sums the entries it wrote: rows 4rg+i, keys kg+16u
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ri = 4 * rg + i;
        float dsum = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) dsum = fmaf(s_p[ri * PS + kg + 16 * u], s_ds[ri * PS + kg + 16 * u], dsum);
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, off);
        if (kg == 0) s_delta[ri] += dsum;
      }
    }
    float aq[EQ];
#pragma unroll
    for (int u = 0; u < EQ; ++u) aq[u] = 0.f;
    // pass 2: dS; drq; dgk, dgv (this CTA's key tiles)
    for (int kt = kgrp; kt < n_kt; kt += n_kg) {
      const int j0 = kt * kLatKeys;
      __syncthreads();
      if (!ONE && n_kt > 1) {  // one tile: its P, dP are still in s_p / s_ds
        load_keys(j0);
        __syncthreads();
        tile_pdp(j0);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ri = 4 * rg + i;
        const float dlt = s_delta[ri];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float* q = s_ds + ri * PS + kg + 16 * u;
          *q = s_p[ri * PS + kg + 16 * u] * (*q - dlt);
        }
      }
      __syncthreads();
      // drq: row `own`, e-quarter eq
#pragma unroll 4
      for (int j = 0; j < kLatKeys; ++j) {
        const float dsv = s_ds[own * PS + j];
        const float* kr = s_k + j * LS + eq * EQ;
#pragma unroll
        for (int u = 0; u < EQ; u += 4) {
          const float4 k4 = *reinterpret_cast<const float4*>(kr + u);
          aq[u] = fmaf(dsv, k4.x, aq[u]);
          aq[u + 1] = fmaf(dsv, k4.y, aq[u + 1]);
          aq[u + 2] = fmaf(dsv, k4.z, aq[u + 2]);
          aq[u + 3] = fmaf(dsv, k4.w, aq[u + 3]);
        }
      }
      // dgk, dgv: key `own` of this tile, e-quarter eq
      float ak[EQ], av[EQ];
#pragma unroll
      for (int u = 0; u < EQ; ++u) ak[u] = av[u] = 0.f;
#pragma unroll 4
      for (int r = 0; r < kLatRows; ++r) {
        const float dsv = s_ds[r * PS + own], pv = s_p[r * PS + own];
        const float* qr = s_rq + r * LS + eq * EQ;
        const float* lr = s_dl + r * LS + eq * EQ;
#pragma unroll
        for (int u = 0; u < EQ; u += 4) {
          const float4 q4 = *reinterpret_cast<const float4*>(qr + u);
          const float4 l4 = *reinterpret_cast<const float4*>(lr + u);
          ak[u] = fmaf(dsv, q4.x, ak[u]);
          ak[u + 1] = fmaf(dsv, q4.y, ak[u + 1]);
          ak[u + 2] = fmaf(dsv, q4.z, ak[u + 2]);
          ak[u + 3] = fmaf(dsv, q4.w, ak[u + 3]);
          av[u] = fmaf(pv, l4.x, av[u]);
          av[u + 1] = fmaf(pv, l4.y, av[u + 1]);
          av[u + 2] = fmaf(pv, l4.z, av[u + 2]);
          av[u + 3] = fmaf(pv, l4.w, av[u + 3]);
        }
      }
      const int j = j0 + own;
      if (ONE) {
#pragma unroll
        for (int u = 0; u < EQ; ++u) {
          ak1[u] += ak[u];
          av1[u] += av[u];
        }
      } else if (j < g.Nc) {
#pragma unroll
        for (int u = 0; u < EQ; ++u) {
          const int e = eq * EQ + u;
          if (e < g.ldh) {
            my_part[(int64_t)(2 * j) * g.Ld + e] += ak[u] * g.lat_scale;
            my_part[(int64_t)(2 * j + 1) * g.Ld + e] += av[u];
          }
        }
      }
    }
    const int r = r0 + own;
    if (r < g.Tq) {
#pragma unroll
      for (int u = 0; u < EQ; ++u) {
        const int e = eq * EQ + u;
        if (e < g.ldh) {
          const int64_t o = ((int64_t)(b * g.Tq + r) * g.Lh + lh) * g.ldh + e;
          if (n_kg > 1)
            drq_part[(int64_t)kgrp * g.B * g.Tq * g.Ld + o] = aq[u] * g.lat_scale;
          else
            drq[o] = from_f<T>(aq[u] * g.lat_scale);
        }
      }
    }
  }
  if (ONE && own < g.Nc) {
#pragma unroll
    for (int u = 0; u < EQ; ++u) {
      const int e = eq * EQ + u;
      if (e < g.ldh) {
        my_part[(int64_t)(2 * own) * g.Ld + e] = ak1[u] * g.lat_scale;
        my_part[(int64_t)(2 * own + 1) * g.Ld + e] = av1[u];
      }
    }
  }
}

// Forward, blocked: a CTA per (64-row block, latent head, b), 256 threads.
// Per 64-key tile: S = rq gk^T as 4-row x 4-key register blocks over float4
// shared-memory operands (the layout of the backward), online softmax in
// log2 units (row max / sum across the 16 threads of a row by shuffles), P
// through shared memory, then O += P gv with each thread owning one row and a
// quarter of the columns. lat_lse = m + ln(l) (natural log) as the backward
// expects; rows that see no chunk (qid = 0) output 0 (models.py:366-373).
template <typename T, int L>
__global__ void __launch_bounds__(256) latent_fwd_blocked_kernel(Geom g, const T* __restrict__ rq,
                                                                 const T* __restrict__ gkv, T* __restrict__ lat,
                                                                 float* __restrict__ lat_lse) {
  using S = LatBwdSmem<L>;
  constexpr int LS = S::LS, PS = S::PS, EQ = L / 4;
  extern __shared__ float4 smem_latf4[];
  float* sm = reinterpret_cast<float*>(smem_latf4);
  float *s_rq = sm + S::RQ, *s_k = sm + S::K, *s_v = sm + S::V, *s_p = sm + S::P;
  float* s_alpha = sm + S::LSE;   // per row: rescale of the running output for this tile
  float* s_l = sm + S::DELTA;     // per row: final normaliser
  int* s_qid = reinterpret_cast<int*>(sm + S::QID);
  const int b = blockIdx.z, lh = blockIdx.y, r0 = blockIdx.x * kLatRows, tid = threadIdx.x;
  const int rg = tid >> 4, kg = tid & 15;  // S block: rows 4rg + i, keys kg + 16u
  const int own = tid >> 2, eq = tid & 3;  // output row and e-quarter
  const float sc2 = g.lat_scale * kLatLog2e;

  for (int idx = tid; idx < kLatRows * L; idx += 256) {
    const int i = idx / L, e = idx % L, r = r0 + i;
    float a = 0.f;
    if (r < g.Tq && e < g.ldh) a = to_f<T>(rq[((int64_t)(b * g.Tq + r) * g.Lh + lh) * g.ldh + e]) * sc2;
    s_rq[i * LS + e] = a;
  }
  if (tid < kLatRows) s_qid[tid] = r0 + tid < g.Tq ? row_qid(g, r0 + tid) : 0;
  const int jmax = row_qid(g, min(r0 + kLatRows - 1, g.Tq - 1));
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
  }
  float acc[EQ];
#pragma unroll
  for (int u = 0; u < EQ; ++u) acc[u] = 0.f;

  for (int j0 = 0; j0 < jmax; j0 += kLatKeys) {
    __syncthreads();
    for (int idx = tid; idx < kLatKeys * L; idx += 256) {
      const int jj = idx / L, e = idx % L, j = j0 + jj;
      float kv = 0.f, vv = 0.f;
      if (j < g.Nc && e < g.ldh) {
        const int64_t base = ((int64_t)(b * g.Nc + j) * 2 * g.Lh + lh) * g.ldh + e;
        kv = to_f<T>(gkv[base]);
        vv = to_f<T>(gkv[base + (int64_t)g.Lh * g.ldh]);
      }
      s_k[jj * LS + e] = kv;
      s_v[jj * LS + e] = vv;
    }
    __syncthreads();
    float sa[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int u = 0; u < 4; ++u) sa[i][u] = 0.f;
#pragma unroll
    for (int e = 0; e < L; e += 4) {
      float4 a[4], k[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = *reinterpret_cast<const float4*>(s_rq + (4 * rg + i) * LS + e);
        k[i] = *reinterpret_cast<const float4*>(s_k + (kg + 16 * i) * LS + e);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          sa[i][u] = fmaf(a[i].x, k[u].x, fmaf(a[i].y, k[u].y, fmaf(a[i].z, k[u].z, fmaf(a[i].w, k[u].w, sa[i][u]))));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ri = 4 * rg + i, qid = s_qid[ri];
      float tm = -INFINITY;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (j0 + kg + 16 * u >= qid) sa[i][u] = -INFINITY;
        tm = fmaxf(tm, sa[i][u]);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
      const float mn = fmaxf(m[i], tm);
      const float alpha = m[i] == -INFINITY ? 0.f : exp2f(m[i] - mn);
      float ps = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float p = sa[i][u] == -INFINITY ? 0.f : exp2f(sa[i][u] - mn);
        s_p[ri * PS + kg + 16 * u] = p;
        ps += p;
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[i] = l[i] * alpha + ps;
      m[i] = mn;
      if (kg == 0) s_alpha[ri] = alpha;
    }
    __syncthreads();
    const float al = s_alpha[own];
#pragma unroll
    for (int u = 0; u < EQ; ++u) acc[u] *= al;
#pragma unroll 4
    for (int j = 0; j < kLatKeys; ++j) {
      const float p = s_p[own * PS + j];
      const float* vr = s_v + j * LS + eq * EQ;
#pragma unroll
      for (int u = 0; u < EQ; u += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(vr + u);
        acc[u] = fmaf(p, v4.x, acc[u]);
        acc[u + 1] = fmaf(p, v4.y, acc[u + 1]);
        acc[u + 2] = fmaf(p, v4.z, acc[u + 2]);
        acc[u + 3] = fmaf(p, v4.w, acc[u + 3]);
      }
    }
  }
  __syncthreads();
  if (kg == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = r0 + 4 * rg + i;
      s_l[4 * rg + i] = l[i];
      if (r < g.Tq) {
        const bool any = s_qid[4 * rg + i] > 0;
        lat_lse[(int64_t)(b * g.Lh + lh) * g.Tq + r] = any ? (m[i] + log2f(l[i])) * 0.6931471805599453f : INFINITY;
      }
    }
  }
  __syncthreads();
  const int r = r0 + own;
  if (r < g.Tq) {
    const float inv = s_qid[own] > 0 ? 1.f / s_l[own] : 0.f;
    T* dst = lat + (int64_t)(b * g.Tq + r) * g.Ld + lh * g.ldh;
#pragma unroll
    for (int u = 0; u < EQ; ++u) {
      const int e = eq * EQ + u;
      if (e < g.ldh) dst[e] = from_f<T>(acc[u] * inv);
    }
  }
}

// out[i] = sum_p part[p * n + i], p in a fixed order (deterministic). A block
// takes 32 consecutive outputs; its 8 warps split the partials (warp w sums
// p = w, w+8, ...) and the 8 sums are added in warp order, so long partial
// lists do not make one thread walk them all.
template <typename To>
__global__ void __launch_bounds__(256) reduce_parts_kernel(const float* __restrict__ part, int n_part, int64_t n,
                                                           To* __restrict__ out) {
  __shared__ float red[8][33];
  const int c = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int64_t i0 = (int64_t)blockIdx.x * 32; i0 < n; i0 += (int64_t)gridDim.x * 32) {
    const int64_t i = i0 + c;
    float a = 0.f;
    if (i < n) {
#pragma unroll 4
      for (int p = w; p < n_part; p += 8) a += part[(int64_t)p * n + i];
    }
    red[w][c] = a;
    __syncthreads();
    if (w == 0 && i < n) {
      float s = red[0][c];
#pragma unroll
      for (int k = 1; k < 8; ++k) s += red[k][c];
      out[i] = from_f<To>(s);
    }
    __syncthreads();
  }
}

template <typename T, int L>
cudaError_t latent_fwd_l(const Geom& g, const T* rq, const T* gkv, T* lat, float* lse, cudaStream_t s) {
  const int sm = (int)sizeof(float) * LatBwdSmem<L>::FLOATS;
  cudaError_t e = set_smem_once(latent_fwd_blocked_kernel<T, L>, sm);
  if (e != cudaSuccess) return e;
  dim3 grid(cdiv(g.Tq, kLatRows), g.Lh, g.B);
  latent_fwd_blocked_kernel<T, L><<<grid, 256, sm, s>>>(g, rq, gkv, lat, lse);
  return cudaGetLastError();
}

template <typename T, int L>
cudaError_t latent_bwd_l(const Geom& g, const T* rq, const T* gkv, const float* lse, const float* dlat, T* drq,
                         float* part, int n_split, int n_kg, float* drq_part, cudaStream_t s) {
  const int sm = (int)sizeof(float) * LatBwdSmem<L>::FLOATS;
  auto k = g.Nc <= kLatKeys ? latent_bwd_kernel<T, L, true> : latent_bwd_kernel<T, L, false>;
  cudaError_t e = set_smem_once(k, sm);
  if (e != cudaSuccess) return e;
  if (g.Nc <= kLatKeys) n_kg = 1;  // one key tile: nothing to split
  dim3 grid(n_split * n_kg, g.Lh, g.B);
  k<<<grid, 256, sm, s>>>(g, rq, gkv, lse, dlat, drq, part, n_split, n_kg, drq_part);
  cudaError_t e2 = cudaGetLastError();
  if (e2 != cudaSuccess || n_kg == 1) return e2;
  return launch_reduce_parts<T>(drq_part, n_kg, (int64_t)g.B * g.Tq * g.Ld, drq, s);
}

}  // namespace

template <typename T>
cudaError_t launch_latent_fwd(const Geom& g, const T* rq, const T* gkv, T* lat, float* lat_lse,
                              cudaStream_t s) {
  if (g.ldh <= 8) return latent_fwd_l<T, 8>(g, rq, gkv, lat, lat_lse, s);
  if (g.ldh <= 16) return latent_fwd_l<T, 16>(g, rq, gkv, lat, lat_lse, s);
  if (g.ldh <= 32) return latent_fwd_l<T, 32>(g, rq, gkv, lat, lat_lse, s);
  return latent_fwd_l<T, 64>(g, rq, gkv, lat, lat_lse, s);
}

template <typename T>
cudaError_t launch_latent_bwd(const Geom& g, const T* rq, const T* gkv, const float* lat_lse, const float* dlat,
                              T* drq, float* dgkv_part, int n_split, int n_kg, float* drq_part, cudaStream_t s) {
  if (g.ldh <= 8) return latent_bwd_l<T, 8>(g, rq, gkv, lat_lse, dlat, drq, dgkv_part, n_split, n_kg, drq_part, s);
  if (g.ldh <= 16) return latent_bwd_l<T, 16>(g, rq, gkv, lat_lse, dlat, drq, dgkv_part, n_split, n_kg, drq_part, s);
  if (g.ldh <= 32) return latent_bwd_l<T, 32>(g, rq, gkv, lat_lse, dlat, drq, dgkv_part, n_split, n_kg, drq_part, s);
  return latent_bwd_l<T, 64>(g, rq, gkv, lat_lse, dlat, drq, dgkv_part, n_split, n_kg, drq_part, s);
}

template <typename T>
cudaError_t launch_latent_reduce(const Geom& g, const float* part, int n_split, T* dgkv,
                                 cudaStream_t s) {
  const int64_t n = (int64_t)g.B * g.Nc * 2 * g.Ld;
  const int blocks = (int)std::min<int64_t>((n + 31) / 32, 148 * 8);
  reduce_parts_kernel<T><<<blocks, 256, 0, s>>>(part, n_split, n, dgkv);
  return cudaGetLastError();
}

cudaError_t launch_reduce_rows(const float* part, int n_part, int64_t n, float* out, cudaStream_t s) {
  return launch_reduce_parts<float>(part, n_part, n, out, s);
}

template <typename To>
cudaError_t launch_reduce_parts(const float* part, int n_part, int64_t n, To* out, cudaStream_t s) {
  const int blocks = (int)std::min<int64_t>((n + 31) / 32, 148 * 8);
  reduce_parts_kernel<To><<<blocks, 256, 0, s>>>(part, n_part, n, out);
  return cudaGetLastError();
}
template cudaError_t launch_reduce_parts<float>(const float*, int, int64_t, float*, cudaStream_t);
template cudaError_t launch_reduce_parts<bf16>(const float*, int, int64_t, bf16*, cudaStream_t);

template cudaError_t launch_latent_fwd<float>(const Geom&, const float*, const float*, float*, float*, cudaStream_t);
template cudaError_t launch_latent_fwd<bf16>(const Geom&, const bf16*, const bf16*, bf16*, float*, cudaStream_t);
template cudaError_t launch_latent_bwd<float>(const Geom&, const float*, const float*, const float*, const float*,
                                              float*, float*, int, int, float*, cudaStream_t);
template cudaError_t launch_latent_bwd<bf16>(const Geom&, const bf16*, const bf16*, const float*, const float*,
                                             bf16*, float*, int, int, float*, cudaStream_t);
template cudaError_t launch_latent_reduce<float>(const Geom&, const float*, int, float*, cudaStream_t);
template cudaError_t launch_latent_reduce<bf16>(const Geom&, const float*, int, bf16*, cudaStream_t);

}  // namespace llattn
