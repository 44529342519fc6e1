// C ABI of libllattn (declared in include/llattn.h): host-side validation,
// geometry, backward workspace layout and kernel dispatch. No device
// allocation and no host synchronisation on the launch paths. Global state:
// the device fault word of the tensor-core kernels, its host-mapped mirror
// (one pinned word per process) and the scratch array of llattn_bwd_noalloc.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "profile.cuh"
#include "sm100.cuh"

namespace llattn {
namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LLATTN_OK;
  return fail(LLATTN_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

// models.py:175-183 (cs, Nc), :249 (bsL), :216-219 (bs, Tq).
int make_geom(const llattn_dims* d, Geom* g) {
  if (!d) return fail(LLATTN_ERR_ARG, "dims is NULL");
  if (d->batch < 1 || d->seq_len < 1) return fail(LLATTN_ERR_ARG, "batch and seq_len must be >= 1");
  if (d->seq_len > 65535) return fail(LLATTN_ERR_ARG, "seq_len %d exceeds 65535", d->seq_len);
  if (d->n_heads < 1 || d->head_dim < 1 || d->head_dim > 128)
    return fail(LLATTN_ERR_ARG, "n_heads >= 1 and 1 <= head_dim <= 128 required (head_dim=%d)", d->head_dim);
  if (d->latent_heads < 1 || d->latent_head_dim < 1 || d->latent_head_dim > 64)
    return fail(LLATTN_ERR_ARG, "latent_heads >= 1 and 1 <= latent_head_dim <= 64 required");
  if (d->latent_heads * d->latent_head_dim > 4096)
    return fail(LLATTN_ERR_ARG, "latent_d_model = %d exceeds 4096", d->latent_heads * d->latent_head_dim);
  if (d->window < 1) return fail(LLATTN_ERR_ARG, "local_window must be positive");
  if (d->latent_tokens < 1) return fail(LLATTN_ERR_ARG, "latent_tokens must be positive");
  if (d->dtype != LLATTN_F32 && d->dtype != LLATTN_BF16) return fail(LLATTN_ERR_ARG, "unknown dtype %d", d->dtype);
  if ((int64_t)d->n_heads * d->head_dim > (1 << 20)) return fail(LLATTN_ERR_ARG, "d_model too large");
  const int T = d->seq_len;
  const int TT = d->total_len > 0 ? d->total_len : T;
  if (d->seq_offset < 0 || (int64_t)d->seq_offset + T > TT)
    return fail(LLATTN_ERR_ARG, "seq_offset %d + seq_len %d exceeds total_len %d", d->seq_offset, T, TT);
  g->off = d->seq_offset;
  g->T_total = TT;
  g->B = d->batch;
  g->T = T;
  g->H = d->n_heads;
  g->hd = d->head_dim;
  g->d = d->n_heads * d->head_dim;
  g->Lh = d->latent_heads;
  g->ldh = d->latent_head_dim;
  g->Ld = d->latent_heads * d->latent_head_dim;
  g->W = d->window;
  g->bsL = std::min(TT, std::max(d->window, d->local_block));
  const int target = std::min(d->latent_tokens, TT);
  g->cs = cdiv(TT, target);
  g->Nc = cdiv(TT, g->cs);
  g->qbs = d->query_block > 1 ? std::min(TT, d->query_block) : 1;
  if (g->off % g->qbs)
    return fail(LLATTN_ERR_ARG, "seq_offset %d must be a multiple of the query block %d", g->off, g->qbs);
  g->Tq = cdiv(T, g->qbs);
  const int d3 = 3 * d->n_heads * d->head_dim;
  g->ldq = d->qkv_row_stride > 0 ? d->qkv_row_stride : d3;
  g->ldd = d->dqkv_row_stride > 0 ? d->dqkv_row_stride : d3;
  if (g->ldq < d3 || g->ldd < d3)
    return fail(LLATTN_ERR_ARG, "qkv / dqkv row strides (%d, %d) below 3 * d_model = %d", g->ldq, g->ldd, d3);
  if (d->dtype == LLATTN_BF16 && ((g->ldq != d3 && g->ldq % 8) || (g->ldd != d3 && g->ldd % 8)))
    return fail(LLATTN_ERR_ARG, "bf16 qkv / dqkv row strides must be multiples of 8");
  g->gate_bias = d->gate_bias;
  g->scale = 1.0f / sqrtf((float)g->hd);
  g->lat_scale = 1.0f / sqrtf((float)g->ldh);
  g->fault_host = nullptr;
  return LLATTN_OK;
}

// Backward workspace, every region 256-byte aligned.
struct BwdLayout {
  size_t dl, delta, drow, drow_half, dlat, dlat_tok, dg_part, dg_sum, dw_part, dgkv_part, drq_part, lat_delta, dbqkv,
      total;
  int gate_tok, n_gate_cta, n_split_w, n_split_lat, n_kg_lat, n_split_keys;
};

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

BwdLayout bwd_layout(const Geom& g, int elt) {
  BwdLayout L;
  L.gate_tok = 16;
  L.n_gate_cta = g.B * cdiv(g.T, L.gate_tok);
  const int rows = g.B * g.Tq;
  // token splits of the dW_rout reduction (enough CTAs to fill the GPU)
  L.n_split_w = std::max(1, std::min(cdiv(g.B * g.T, 64), (2 * 148) / cdiv(g.d, 128)));
  // row splits of the latent backward: (b, latent head, split) CTAs, about two per SM
  L.n_split_lat = std::max(1, std::min(cdiv(g.Tq, 64), (2 * 148) / (g.B * g.Lh)));
  // SIMT latent backward with several 64-key tiles and too few row splits
  // to fill the GPU: split the key tiles of each row split over CTAs
  {
    const int base = g.B * g.Lh * L.n_split_lat, n_kt = cdiv(g.Nc, 64);
    L.n_kg_lat = (n_kt > 1 && base < 148) ? std::max(1, std::min(n_kt, (2 * 148) / base)) : 1;
  }
  // row splits of the tensor-core latent keys kernel (64 < Nc <= 512): one
  // CTA per SM, about two waves of (128-key tile, split, latent head, b)
  L.n_split_keys = std::max(1, std::min(cdiv(g.Tq, 64), (2 * 148) / (g.B * g.Lh * cdiv(g.Nc, 128))));
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  const size_t BTd = (size_t)g.B * g.T * g.d;
  L.dl = take(BTd * elt);
  L.delta = take(sizeof(float) * g.B * g.H * g.T);
  // fp32 dremote (SIMT), bf16 dR (fused tensor-core path), or the general
  // path's bf16 remote rows [B*Tq, d] and, from drow_half on, its dR rows
  L.drow_half = align256(sizeof(bf16) * (size_t)g.B * g.Tq * g.d);
  L.drow = take(std::max(sizeof(float) * BTd, 2 * L.drow_half));
  L.dlat = take(sizeof(float) * (size_t)rows * g.Ld);
  L.dlat_tok = take(sizeof(float) * (size_t)g.B * g.T * g.Ld);
  // dg partials: [n_gate_cta][2 hd] (SIMT gate) or [gate_bwd_ctas][hd + 65 H] (tensor-core gate)
  const size_t dg_tc = (size_t)g.B * cdiv(g.T, 128) * (g.hd + 65 * g.H);
  const size_t dg_rm = (size_t)g.B * std::max(cdiv(g.T, 16), g.Tq) * 2 * g.hd;  // general path's gate CTAs
  L.dg_part = take(sizeof(float) * std::max(std::max((size_t)L.n_gate_cta * 2 * g.hd, dg_tc), dg_rm));
  L.dg_sum = take(sizeof(float) * (size_t)std::max(2 * g.hd, g.hd + 65 * g.H));
  L.dw_part = take(sizeof(float) * (size_t)L.n_split_w * g.d * (g.Ld + 1));
  const bool long_lat = g.Nc > 64;
  L.dgkv_part = take(sizeof(float) * (size_t)std::max(L.n_split_lat * L.n_kg_lat, long_lat ? L.n_split_keys : 0) *
                     g.B * g.Nc * 2 * g.Ld);
  L.drq_part = take(L.n_kg_lat > 1 ? sizeof(float) * (size_t)L.n_kg_lat * g.B * g.Tq * g.Ld : 0);
  L.lat_delta = take(long_lat ? sizeof(float) * (size_t)g.B * g.Lh * g.Tq : 0);
  // qkv_proj bias gradient: the column-sum kernel's split partials
  L.dbqkv = take(sizeof(float) * 3 * (size_t)g.d * colsum_splits((int64_t)g.B * g.T, 3 * g.d, elt));
  L.total = off;
  return L;
}

bool al(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

std::mutex g_attr_mu;
struct AttrEntry {
  const void* kernel;
  int dev, bytes;
};
AttrEntry g_attr[512];
int g_n_attr = 0;

}  // namespace

cudaError_t set_smem_attr(const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  for (int i = 0; i < g_n_attr; ++i)
    if (g_attr[i].kernel == kernel && g_attr[i].dev == dev) {
      if (g_attr[i].bytes >= bytes) return cudaSuccess;
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (e == cudaSuccess) g_attr[i].bytes = bytes;
      return e;
    }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && g_n_attr < 512) g_attr[g_n_attr++] = {kernel, dev, bytes};
  return e;
}

namespace {

// Host-mapped fault word: a tensor-core kernel whose bounded wait runs out
// sets it (besides the device word that stops the other CTAs), and every
// launching entry point tests it first, without synchronising. A fault thus
// surfaces as LLATTN_ERR_DEVICE at the next call, the way CUDA reports an
// asynchronous error, instead of later calls silently returning the outputs
// of kernels that exit at once on the sticky device word.
std::mutex g_fault_mu;
volatile unsigned* g_fault_host = nullptr;

volatile unsigned* fault_host_word() {
  std::lock_guard<std::mutex> lk(g_fault_mu);
  if (!g_fault_host) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, 64, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    *static_cast<volatile unsigned*>(p) = 0u;
    g_fault_host = static_cast<volatile unsigned*>(p);
  }
  return g_fault_host;
}

// Before a launch: attach the mirror to the geometry and refuse to run once
// a fault has been recorded (cleared by llattn_fault_status(1)).
int fault_gate(Geom* g) {
  volatile unsigned* w = fault_host_word();
  if (!w) return fail(LLATTN_ERR_LAUNCH, "cannot allocate the host-mapped fault word");
  const unsigned bits = *w;
  if (bits)
    return fail(LLATTN_ERR_DEVICE,
                "an earlier tensor-core launch gave up on a barrier wait (fault bits 0x%x); its outputs and "
                "those of the launches queued after it are invalid. llattn_fault_status(1) clears the fault",
                bits);
  void* dp = nullptr;
  if (cudaHostGetDevicePointer(&dp, const_cast<unsigned*>(w), 0) != cudaSuccess) {
    cudaGetLastError();
    return fail(LLATTN_ERR_LAUNCH, "the fault word is not mapped for the current device");
  }
  g->fault_host = static_cast<volatile unsigned*>(dp);
  return LLATTN_OK;
}

// The general tensor-core path needs 16-byte rows for the GEMM's copies.
bool general_ok(const Geom& g) { return g.Ld % 8 == 0 && g.d % 8 == 0 && g.hd % 4 == 0; }

// The SIMT r_out / gate kernels hold at most 128 latent columns per row.
int simt_gate_check(const Geom& g) {
  if (g.Ld > 128)
    return fail(LLATTN_ERR_ARG,
                "latent_d_model = %d > 128 needs the tensor-core path (bf16 activations, head_dim 64 or 128, "
                "latent_d_model a multiple of 8)",
                g.Ld);
  return LLATTN_OK;
}

// Tensor-core path for geometries the fused gate epilogue does not hold
// (latent_d_model != 64, or more than 32 heads): local forward without the
// epilogue, remote = lat W_rout^T + b_rout by the tensor-core GEMM written
// into the rows of `mixed` the gate kernel reads them from, then gate and
// mix in place.
int run_fwd_general(const Geom& g, const llattn_fwd_args* a, cudaStream_t s) {
  int rc;
  {
    prof::Scope ps(prof::LOCAL_FWD, s);
    sm100::GateEpilogue ep{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    rc = check_launch(sm100::launch_local_fwd(g, a->qkv, a->local_out, a->lse, ep, s), "local_fwd_sm100");
  }
  if (rc) return rc;
  prof::Scope ps(prof::GATE_FWD, s, 2);
  sm100::GemmOut o{};
  o.C = a->mixed;
  o.ldc = g.d;
  o.out_bf16 = 1;
  o.bias = a->b_rout;
  o.rows_per_group = g.Tq;
  o.group_stride = g.T;
  o.row_step = g.qbs;
  rc = check_launch(sm100::launch_gemm(g, g.B * g.Tq, g.d, g.Ld, a->lat, g.Ld, 0, a->w_rout, g.Ld, 0, o, 1, s),
                    "remote_gemm");
  if (rc) return rc;
  return check_launch(launch_gate_mix_rmem(g, static_cast<const bf16*>(a->local_out), a->g_local, a->g_remote,
                                           static_cast<bf16*>(a->mixed), s),
                      "gate_mix");
}

template <typename T>
int run_fwd(const Geom& g, const llattn_fwd_args* a, cudaStream_t s) {
  const T* qkv = static_cast<const T*>(a->qkv);
  const bool tc = sm100::fwd_supported(g, sizeof(T));
  const bool fused = tc && sm100::gate_fusable(g);
  const bool general = tc && !fused && general_ok(g);
  int rc;
  if (!fused && !general && (rc = simt_gate_check(g))) return rc;
  {
    prof::Scope ps(prof::LATENT_FWD, s);
    if (sizeof(T) == 2 && sm100::latent_tc_fwd_ok(g))  // tensor cores: bf16, head dim <= 64, <= 512 chunks
      rc = check_launch(sm100::launch_latent_fwd_tc(g, a->rq, a->gkv, a->lat, a->lat_lse, s), "latent_fwd_sm100");
    else
      rc = check_launch(launch_latent_fwd<T>(g, static_cast<const T*>(a->rq), static_cast<const T*>(a->gkv),
                                             static_cast<T*>(a->lat), a->lat_lse, s),
                        "latent_fwd");
  }
  if (rc) return rc;
  if (general) return run_fwd_general(g, a, s);
  {
  prof::Scope ps(prof::LOCAL_FWD, s);
  if (tc) {
    sm100::GateEpilogue ep{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    if (fused) ep = {a->lat, a->w_rout, a->b_rout, a->g_local, a->g_remote, a->mixed};
    rc = check_launch(sm100::launch_local_fwd(g, a->qkv, a->local_out, a->lse, ep, s), "local_fwd_sm100");
  } else {
    rc = check_launch(launch_local_fwd_simt<T>(g, qkv, static_cast<T*>(a->local_out), a->lse, s),
                      "local_fwd_simt");
  }
  }
  if (rc || fused) return rc;
  prof::Scope ps(prof::GATE_FWD, s);
  return check_launch(launch_gate_fwd<T>(g, static_cast<const T*>(a->local_out), static_cast<const T*>(a->lat),
                                         static_cast<const T*>(a->w_rout), a->b_rout, a->g_local, a->g_remote,
                                         static_cast<T*>(a->mixed), s),
                      "gate_fwd");
}

template <typename T>
int run_bwd(const Geom& g, const llattn_bwd_args* a, cudaStream_t s) {
  int rc0;
  const BwdLayout L = bwd_layout(g, sizeof(T));
  char* ws = static_cast<char*>(a->workspace);
  T* dl = reinterpret_cast<T*>(ws + L.dl);
  float* delta = reinterpret_cast<float*>(ws + L.delta);
  float* drow = reinterpret_cast<float*>(ws + L.drow);
  float* dlat = reinterpret_cast<float*>(ws + L.dlat);
  float* dg_part = reinterpret_cast<float*>(ws + L.dg_part);
  float* dg_sum = reinterpret_cast<float*>(ws + L.dg_sum);
  float* dw_part = reinterpret_cast<float*>(ws + L.dw_part);
  float* dgkv_part = reinterpret_cast<float*>(ws + L.dgkv_part);
  const T* lat = static_cast<const T*>(a->lat);
  const T* w_rout = static_cast<const T*>(a->w_rout);

  const bool tc = sm100::bwd_supported(g, sizeof(T)) && sm100::gate_fusable(g);
  const bool general =
      sizeof(T) == 2 && sm100::bwd_supported(g, sizeof(T)) && !sm100::gate_fusable(g) && general_ok(g);
  if (!tc && !general && (rc0 = simt_gate_check(g))) return rc0;
  int n_dg = L.n_gate_cta;
  int rc;
  if (general) {
    // remote rows recomputed by the GEMM, the gate backward on them, the
    // local backward, then dlat = dR W_rout, dW_rout = dR^T lat and db_rout
    // (column sums) by the GEMM, with dR per query row (summed over each
    // query block for block-pooled queries)
    bf16* rem = reinterpret_cast<bf16*>(ws + L.drow);
    bf16* dr = reinterpret_cast<bf16*>(ws + L.drow + L.drow_half);
    const int rows = g.B * g.Tq;
    n_dg = gate_rmem_ctas(g);
    {
      prof::Scope ps(prof::GATE_BWD, s, 2);
      sm100::GemmOut o{};
      o.C = rem;
      o.ldc = g.d;
      o.out_bf16 = 1;
      o.bias = a->b_rout;
      rc = check_launch(sm100::launch_gemm(g, rows, g.d, g.Ld, a->lat, g.Ld, 0, a->w_rout, g.Ld, 0, o, 1, s),
                        "remote_gemm");
      if (rc) return rc;
      rc = check_launch(launch_gate_bwd_rmem(g, static_cast<const bf16*>(a->local_out), rem, a->g_local,
                                             a->g_remote, static_cast<const bf16*>(a->dmixed),
                                             reinterpret_cast<bf16*>(dl), delta, dr, dg_part, s),
                        "gate_bwd_rmem");
    }
    if (rc) return rc;
    {
      prof::Scope ps(prof::LOCAL_DQ, s);
      rc = check_launch(sm100::launch_local_dq(g, a->qkv, dl, a->lse, delta, a->dqkv, s), "local_dq_sm100");
    }
    if (rc) return rc;
    {
      prof::Scope ps(prof::LOCAL_DKV, s);
      rc = check_launch(sm100::launch_local_dkv(g, a->qkv, dl, a->lse, delta, a->dqkv, s), "local_dkv_sm100");
    }
    if (rc) return rc;
    {
      prof::Scope ps(prof::ROUT_BWD, s, 2);
      sm100::GemmOut o{};
      o.C = dlat;
      o.ldc = g.Ld;
      rc = check_launch(sm100::launch_gemm(g, rows, g.Ld, g.d, dr, g.d, 0, a->w_rout, g.Ld, 1, o, 1, s),
                        "dlat_gemm");
      if (rc) return rc;
      sm100::GemmOut w{};
      w.C = dw_part;
      w.ldc = g.Ld;
      w.split_stride = (int64_t)g.d * g.Ld;
      w.colsum = dw_part + (size_t)L.n_split_w * g.d * g.Ld;
      w.colsum_split = g.d;
      rc = check_launch(sm100::launch_gemm(g, g.d, g.Ld, rows, dr, g.d, 1, a->lat, g.Ld, 1, w, L.n_split_w, s),
                        "dw_gemm");
      if (rc) return rc;
    }
  } else if (tc) {
    // tensor-core path: gate backward (also dlat, dR bf16, dg partials), then
    // the local backward, then the dW_rout / db_rout GEMM from dR
    bf16* dr = reinterpret_cast<bf16*>(drow);
    float* dlat_tok = reinterpret_cast<float*>(ws + L.dlat_tok);
    n_dg = sm100::gate_bwd_ctas(g);
    {
      prof::Scope ps(prof::GATE_BWD, s);
      sm100::GateBwd gb{a->local_out, a->lat,   a->w_rout, a->b_rout, a->g_local, a->g_remote,
                        a->dmixed,    dl,       delta,     dr,        dlat_tok,   dg_part};
      rc = check_launch(sm100::launch_gate_bwd(g, gb, s), "gate_bwd_sm100");
    }
    if (rc) return rc;
    {
      prof::Scope ps(prof::LOCAL_DQ, s);
      rc = check_launch(sm100::launch_local_dq(g, a->qkv, dl, a->lse, delta, a->dqkv, s), "local_dq_sm100");
    }
    if (rc) return rc;
    {
      prof::Scope ps(prof::LOCAL_DKV, s);
      rc = check_launch(sm100::launch_local_dkv(g, a->qkv, dl, a->lse, delta, a->dqkv, s), "local_dkv_sm100");
    }
    if (rc) return rc;
    {
      prof::Scope ps(prof::ROUT_BWD, s, g.qbs > 1 ? 2 : 1);
      rc = check_launch(sm100::launch_rout_dw(g, dr, a->lat, dw_part, dw_part + (size_t)L.n_split_w * g.d * g.Ld,
                                              L.n_split_w, s),
                        "rout_dw_sm100");
      if (rc) return rc;
      if (g.qbs > 1) {
        rc = check_launch(sm100::launch_dlat_rowsum(g, dlat_tok, dlat, s), "dlat_rowsum");
        if (rc) return rc;
      } else {
        dlat = dlat_tok;
      }
    }
  } else {
  {
  prof::Scope ps(prof::GATE_BWD, s);
  rc = check_launch(
      launch_gate_bwd<T>(g, static_cast<const T*>(a->local_out), lat, w_rout, a->b_rout, a->g_local, a->g_remote,
                         static_cast<const T*>(a->dmixed), dl, delta, drow, dg_part, L.gate_tok, s),
      "gate_bwd");
  }
  if (rc) return rc;
  if (sm100::bwd_supported(g, sizeof(T))) {
    {
      prof::Scope ps(prof::LOCAL_DQ, s);
      rc = check_launch(sm100::launch_local_dq(g, a->qkv, dl, a->lse, delta, a->dqkv, s), "local_dq_sm100");
    }
    if (rc) return rc;
    prof::Scope ps(prof::LOCAL_DKV, s);
    rc = check_launch(sm100::launch_local_dkv(g, a->qkv, dl, a->lse, delta, a->dqkv, s), "local_dkv_sm100");
  } else {
    prof::Scope ps(prof::LOCAL_BWD, s, 2);
    rc = check_launch(launch_local_bwd_simt<T>(g, static_cast<const T*>(a->qkv), dl, a->lse, delta,
                                               static_cast<T*>(a->dqkv), s),
                      "local_bwd_simt");
  }
  if (rc) return rc;
  {
  prof::Scope ps(prof::ROUT_BWD, s, 2);
  rc = check_launch(launch_rout_bwd<T>(g, drow, lat, w_rout, dlat, dw_part, L.n_split_w, s), "rout_bwd");
  }
  if (rc) return rc;
  }
  {
  prof::Scope ps(prof::REDUCE, s, tc ? 4 : 3);
  rc = check_launch(launch_reduce_rows(dw_part, L.n_split_w, (int64_t)g.d * g.Ld, a->dw_rout, s), "reduce_dw");
  if (rc) return rc;
  rc = check_launch(launch_reduce_rows(dw_part + (size_t)L.n_split_w * g.d * g.Ld, L.n_split_w, g.d, a->db_rout, s),
                    "reduce_db");
  if (rc) return rc;
  // dg partials: SIMT [cta][2*hd] (local half, remote half); tensor-core
  // [cta][hd + 65 H] (local, then the S1/S0 sums dg_remote is linear in)
  const int dg_n = tc ? sm100::gate_dg_floats(g) : 2 * g.hd;  // general: the SIMT format
  rc = check_launch(launch_reduce_rows(dg_part, n_dg, dg_n, dg_sum, s), "reduce_dg");
  if (rc) return rc;
  rc = check_launch(cudaMemcpyAsync(a->dg_local, dg_sum, sizeof(float) * g.hd, cudaMemcpyDeviceToDevice, s),
                    "copy dg_local");
  if (rc) return rc;
  if (tc)
    rc = check_launch(sm100::launch_gate_dgr_finalize(g, dg_sum, a->w_rout, a->b_rout, a->dg_remote, s),
                      "gate_dgr_finalize");
  else
    rc = check_launch(cudaMemcpyAsync(a->dg_remote, dg_sum + g.hd, sizeof(float) * g.hd,
                                      cudaMemcpyDeviceToDevice, s),
                      "copy dg_remote");
  }
  if (rc) return rc;
  // tensor-core latent backward for bf16 with head dim <= 64 and <= 64 chunks;
  // its row splits are 128-row tiles, at most the SIMT kernel's 64-row count
  const bool lat_tc = sizeof(T) == 2 && sm100::latent_tc_ok(g);
  // past 64 chunks: the tensor-core rows / keys kernels (up to 512 chunks)
  const bool lat_tc_long = sizeof(T) == 2 && !lat_tc && sm100::latent_tc_long_ok(g);
  const int n_split_lat = lat_tc ? std::min(sm100::latent_tc_splits(g), L.n_split_lat)
                                 : lat_tc_long ? L.n_split_keys : L.n_split_lat;
  const int n_kg_lat = lat_tc || lat_tc_long || g.Nc <= 64 ? 1 : L.n_kg_lat;
  {
  prof::Scope ps(prof::LATENT_BWD, s, n_kg_lat > 1 || lat_tc_long ? 3 : 2);
  if (lat_tc)
    rc = check_launch(sm100::launch_latent_bwd_tc(g, a->rq, a->gkv, a->lat_lse, dlat, a->drq, dgkv_part,
                                                  n_split_lat, s),
                      "latent_bwd_sm100");
  else if (lat_tc_long)
    rc = check_launch(sm100::launch_latent_bwd_tc_long(g, a->rq, a->gkv, a->lat_lse, dlat, a->drq,
                                                       reinterpret_cast<float*>(ws + L.lat_delta), dgkv_part,
                                                       n_split_lat, s),
                      "latent_bwd_sm100_long");
  else
    rc = check_launch(launch_latent_bwd<T>(g, static_cast<const T*>(a->rq), static_cast<const T*>(a->gkv),
                                           a->lat_lse, dlat, static_cast<T*>(a->drq), dgkv_part, n_split_lat,
                                           n_kg_lat, reinterpret_cast<float*>(ws + L.drq_part), s),
                      "latent_bwd");
  if (rc) return rc;
  rc = check_launch(launch_latent_reduce<T>(g, dgkv_part, n_split_lat * n_kg_lat, static_cast<T*>(a->dgkv), s),
                    "latent_reduce");
  }
  if (rc || !a->db_qkv) return rc;
  prof::Scope pc(prof::COLSUM, s, 2);
  return check_launch(launch_colsum<T, float>(static_cast<const T*>(a->dqkv), (int64_t)g.B * g.T, 3 * (int64_t)g.d,
                                              reinterpret_cast<float*>(ws + L.dbqkv), a->db_qkv, s, g.ldd),
                      "colsum_dbqkv");
}

}  // namespace
}  // namespace llattn

using namespace llattn;

extern "C" {

int llattn_version(void) { return LLATTN_VERSION; }

unsigned llattn_fault_status(int reset) {
  unsigned v = sm100::read_fault_word(reset != 0);
  volatile unsigned* w = fault_host_word();
  if (w) {
    v |= *w;
    if (reset) *w = 0u;
  }
  return v;
}

int llattn_fault_inject_host(unsigned bits) {
  volatile unsigned* w = fault_host_word();
  if (!w) return fail(LLATTN_ERR_LAUNCH, "cannot allocate the host-mapped fault word");
  *w |= bits;
  return LLATTN_OK;
}

const char* llattn_last_error(void) { return g_err; }

int llattn_geometry(const llattn_dims* dims, llattn_geom* out) {
  Geom g;
  int rc = make_geom(dims, &g);
  if (rc) return rc;
  if (!out) return fail(LLATTN_ERR_ARG, "out is NULL");
  out->chunk = g.cs;
  out->n_chunks = g.Nc;
  out->local_span = g.bsL;
  out->qblock = g.qbs;
  out->n_qrows = g.Tq;
  return LLATTN_OK;
}

size_t llattn_bwd_workspace_bytes(const llattn_dims* dims) {
  Geom g;
  if (make_geom(dims, &g)) return 0;
  return bwd_layout(g, dims->dtype == LLATTN_BF16 ? 2 : 4).total;
}

int llattn_pool_fwd(const llattn_dims* dims, int mode, const void* x, void* pooled, int64_t d, void* stream) {
  Geom g;
  int rc = make_geom(dims, &g);
  if (rc) return rc;
  if (!x || !pooled) return fail(LLATTN_ERR_ARG, "pool_fwd: NULL pointer");
  if (mode != LLATTN_POOL_CHUNKS && mode != LLATTN_POOL_QBLOCKS) return fail(LLATTN_ERR_ARG, "bad pool mode");
  if (d < 1) return fail(LLATTN_ERR_ARG, "pool_fwd: d must be >= 1");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prof::Scope ps(prof::POOL_FWD, s);
  if (dims->dtype == LLATTN_BF16)
    return check_launch(launch_pool_fwd<bf16>(g, mode, (const bf16*)x, (bf16*)pooled, d, s), "pool_fwd");
  return check_launch(launch_pool_fwd<float>(g, mode, (const float*)x, (float*)pooled, d, s), "pool_fwd");
}

int llattn_pool_bwd(const llattn_dims* dims, int mode, const void* dpooled, void* dx, int64_t d, void* stream) {
  Geom g;
  int rc = make_geom(dims, &g);
  if (rc) return rc;
  if (!dpooled || !dx) return fail(LLATTN_ERR_ARG, "pool_bwd: NULL pointer");
  const int acc = (mode & LLATTN_POOL_ACCUMULATE) ? 1 : 0;
  mode &= ~LLATTN_POOL_ACCUMULATE;
  if (mode != LLATTN_POOL_CHUNKS && mode != LLATTN_POOL_QBLOCKS) return fail(LLATTN_ERR_ARG, "bad pool mode");
  if (d < 1) return fail(LLATTN_ERR_ARG, "pool_bwd: d must be >= 1");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prof::Scope ps(prof::POOL_BWD, s);
  if (dims->dtype == LLATTN_BF16)
    return check_launch(launch_pool_bwd<bf16>(g, mode, (const bf16*)dpooled, (bf16*)dx, d, acc, s), "pool_bwd");
  return check_launch(launch_pool_bwd<float>(g, mode, (const float*)dpooled, (float*)dx, d, acc, s), "pool_bwd");
}

int llattn_pool_proj_fwd(const llattn_dims* dims, const void* z, int64_t ldz, const void* b_rkv, const void* b_rq,
                         void* gkv, void* rq, void* stream) {
  Geom g;
  int rc = make_geom(dims, &g);
  if (rc) return rc;
  if (!z || !gkv || !rq) return fail(LLATTN_ERR_ARG, "pool_proj_fwd: NULL pointer");
  if (g.off != 0 || g.T_total != g.T) return fail(LLATTN_ERR_ARG, "pool_proj_fwd: whole sequences only");
  if (ldz < 3 * (int64_t)g.Ld) return fail(LLATTN_ERR_ARG, "pool_proj_fwd: ldz %lld < 3 * latent_d_model", (long long)ldz);
  if (g.Ld > 128) return fail(LLATTN_ERR_ARG, "pool_proj_fwd: latent_d_model %d > 128", g.Ld);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prof::Scope ps(prof::POOL_FWD, s);
  if (dims->dtype == LLATTN_BF16)
    return check_launch(launch_pool_proj_fwd<bf16>(g, (const bf16*)z, ldz, (const bf16*)b_rkv, (const bf16*)b_rq,
                                                   (bf16*)gkv, (bf16*)rq, s),
                        "pool_proj_fwd");
  return check_launch(launch_pool_proj_fwd<float>(g, (const float*)z, ldz, (const float*)b_rkv, (const float*)b_rq,
                                                  (float*)gkv, (float*)rq, s),
                      "pool_proj_fwd");
}

int llattn_pool_proj_bwd(const llattn_dims* dims, const void* dgkv, const void* drq, void* dz, int64_t ldz,
                         void* stream) {
  Geom g;
  int rc = make_geom(dims, &g);
  if (rc) return rc;
  if (!dgkv || !drq || !dz) return fail(LLATTN_ERR_ARG, "pool_proj_bwd: NULL pointer");
  if (g.off != 0 || g.T_total != g.T) return fail(LLATTN_ERR_ARG, "pool_proj_bwd: whole sequences only");
  if (ldz < 3 * (int64_t)g.Ld) return fail(LLATTN_ERR_ARG, "pool_proj_bwd: ldz %lld < 3 * latent_d_model", (long long)ldz);
  if (g.Ld > 128) return fail(LLATTN_ERR_ARG, "pool_proj_bwd: latent_d_model %d > 128", g.Ld);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prof::Scope ps(prof::POOL_BWD, s);
  if (dims->dtype == LLATTN_BF16)
    return check_launch(launch_pool_proj_bwd<bf16>(g, (const bf16*)dgkv, (const bf16*)drq, (bf16*)dz, ldz, s),
                        "pool_proj_bwd");
  return check_launch(launch_pool_proj_bwd<float>(g, (const float*)dgkv, (const float*)drq, (float*)dz, ldz, s),
                      "pool_proj_bwd");
}

size_t llattn_colsum_workspace_bytes(int64_t rows, int64_t cols, int dtype) {
  if (rows < 1 || cols < 1 || (dtype != LLATTN_BF16 && dtype != LLATTN_F32)) return 0;
  return sizeof(float) * (size_t)colsum_splits(rows, cols, dtype == LLATTN_BF16 ? 2 : 4) * (size_t)cols;
}

int llattn_colsum(const void* g, int64_t rows, int64_t cols, int dtype, void* out, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (!g || !out || !workspace) return fail(LLATTN_ERR_ARG, "colsum: NULL pointer");
  const size_t need = llattn_colsum_workspace_bytes(rows, cols, dtype);
  if (need == 0) return fail(LLATTN_ERR_ARG, "colsum: bad rows, cols or dtype");
  if (cols > (int64_t)INT32_MAX / 32) return fail(LLATTN_ERR_ARG, "colsum: cols too large");
  if (workspace_bytes < need) return fail(LLATTN_ERR_ARG, "colsum: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prof::Scope ps(prof::COLSUM, s, 2);
  if (dtype == LLATTN_BF16)
    return check_launch(launch_colsum<bf16, bf16>((const bf16*)g, rows, cols, (float*)workspace, (bf16*)out, s),
                        "colsum");
  return check_launch(launch_colsum<float, float>((const float*)g, rows, cols, (float*)workspace, (float*)out, s),
                      "colsum");
}

int llattn_fwd(const llattn_fwd_args* a, void* stream) {
  if (!a) return fail(LLATTN_ERR_ARG, "args is NULL");
  Geom g;
  int rc = make_geom(&a->dims, &g);
  if (rc) return rc;
  if (!a->qkv || !a->rq || !a->gkv || !a->w_rout || !a->b_rout || !a->g_local || !a->g_remote || !a->mixed ||
      !a->local_out || !a->lse || !a->lat || !a->lat_lse)
    return fail(LLATTN_ERR_ARG, "llattn_fwd: NULL pointer in args");
  if ((rc = fault_gate(&g))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->dims.dtype == LLATTN_BF16) return run_fwd<bf16>(g, a, s);
  return run_fwd<float>(g, a, s);
}

int llattn_decode(const llattn_decode_args* a, void* stream) {
  if (!a) return fail(LLATTN_ERR_ARG, "args is NULL");
  Geom g;
  int rc = make_geom(&a->dims, &g);
  if (rc) return rc;
  if (!a->qkv_cache || !a->rq_row || !a->gkv || !a->w_rout || !a->b_rout || !a->g_local || !a->g_remote ||
      !a->mixed_row)
    return fail(LLATTN_ERR_ARG, "llattn_decode: NULL pointer in args");
  if (a->cache_len < a->dims.seq_len)
    return fail(LLATTN_ERR_ARG, "llattn_decode: cache_len %lld < seq_len %d", (long long)a->cache_len,
                a->dims.seq_len);
  if ((rc = fault_gate(&g))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prof::Scope ps(prof::DECODE, s);
  if (a->dims.dtype == LLATTN_BF16)
    return check_launch(launch_decode<bf16>(g, a->cache_len, (const bf16*)a->qkv_cache, (const bf16*)a->rq_row,
                                            (const bf16*)a->gkv, (const bf16*)a->w_rout, a->b_rout, a->g_local,
                                            a->g_remote, (bf16*)a->mixed_row, s),
                        "decode");
  return check_launch(launch_decode<float>(g, a->cache_len, (const float*)a->qkv_cache, (const float*)a->rq_row,
                                           (const float*)a->gkv, (const float*)a->w_rout, a->b_rout, a->g_local,
                                           a->g_remote, (float*)a->mixed_row, s),
                      "decode");
}

int llattn_bwd(const llattn_bwd_args* a, void* stream) {
  if (!a) return fail(LLATTN_ERR_ARG, "args is NULL");
  Geom g;
  int rc = make_geom(&a->dims, &g);
  if (rc) return rc;
  if (!a->qkv || !a->rq || !a->gkv || !a->w_rout || !a->b_rout || !a->g_local || !a->g_remote ||
      !a->local_out || !a->lse || !a->lat || !a->lat_lse || !a->dmixed || !a->dqkv || !a->drq || !a->dgkv ||
      !a->dw_rout || !a->db_rout || !a->dg_local || !a->dg_remote)
    return fail(LLATTN_ERR_ARG, "llattn_bwd: NULL pointer in args");
  const size_t need = bwd_layout(g, a->dims.dtype == LLATTN_BF16 ? 2 : 4).total;
  if (!a->workspace || a->workspace_bytes < need)
    return fail(LLATTN_ERR_WORKSPACE, "llattn_bwd: workspace of %zu bytes needed, %zu given", need,
                a->workspace_bytes);
  if (!al(a->workspace, 256)) return fail(LLATTN_ERR_ALIGN, "llattn_bwd: workspace must be 256-byte aligned");
  if ((rc = fault_gate(&g))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->dims.dtype == LLATTN_BF16) return run_bwd<bf16>(g, a, s);
  return run_bwd<float>(g, a, s);
}

// ---------------------------------------------------------------------------
// llattn_bwd_noalloc: the backward for callers that must not allocate device
// memory themselves. Its workspace is this file-scope array, reserved on every
// GPU that loads the library for the life of the process.
static __device__ __align__(256) unsigned char g_bwd_noalloc_scratch[LLATTN_BWD_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64];  // device address of the array, per device

int llattn_bwd_noalloc(const llattn_bwd_args* a, void* stream) {
  if (!a) return fail(LLATTN_ERR_ARG, "args is NULL");
  Geom g;
  int rc = make_geom(&a->dims, &g);
  if (rc) return rc;
  const size_t need = bwd_layout(g, a->dims.dtype == LLATTN_BF16 ? 2 : 4).total;
  if (need > (size_t)LLATTN_BWD_NOALLOC_SCRATCH_BYTES)
    return fail(LLATTN_ERR_WORKSPACE,
                "llattn_bwd_noalloc: these dims need %zu bytes of scratch, more than its fixed %zu bytes; "
                "use llattn_bwd with a caller-provided workspace",
                need, (size_t)LLATTN_BWD_NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(LLATTN_ERR_LAUNCH, "llattn_bwd_noalloc: no usable current device");
  if (stream) {
    // the scratch address is the current device's copy of the array: a
    // stream of another device would run the kernels on that device with
    // a pointer into this one's memory
    int sdev = -1;
    if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess) {
      cudaGetLastError();
      return fail(LLATTN_ERR_ARG, "llattn_bwd_noalloc: cannot query the stream's device");
    }
    if (sdev != dev)
      return fail(LLATTN_ERR_ARG, "llattn_bwd_noalloc: stream belongs to device %d, current device is %d", sdev,
                  dev);
  }
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      // once per device, with that device current: the host-side symbol is
      // only a stand-in, the kernels need the array's device address
      cudaError_t e = cudaGetSymbolAddress(&g_noalloc_ptr[dev], g_bwd_noalloc_scratch);
      if (e != cudaSuccess) {
        g_noalloc_ptr[dev] = nullptr;
        cudaGetLastError();
        // the array is reserved when the library's module loads on the
        // device (first use under lazy loading): that load fails when the
        // device has no 32 MiB left, e.g. under a caching allocator
        if (e == cudaErrorMemoryAllocation)
          return fail(LLATTN_ERR_WORKSPACE,
                      "llattn_bwd_noalloc: device %d has no room for the library's fixed %u-byte scratch array "
                      "(reserved when the library first loads on the device); free device memory first or use "
                      "llattn_bwd with a caller-provided workspace",
                      dev, (unsigned)LLATTN_BWD_NOALLOC_SCRATCH_BYTES);
        return fail(LLATTN_ERR_LAUNCH, "llattn_bwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      }
    }
    ptr = g_noalloc_ptr[dev];
  }
  // Same kernels as llattn_bwd; every workspace region is fully written before
  // it is read, so the array's previous contents never need clearing.
  llattn_bwd_args b = *a;
  b.workspace = ptr;
  b.workspace_bytes = (size_t)LLATTN_BWD_NOALLOC_SCRATCH_BYTES;
  return llattn_bwd(&b, stream);
}

}  // extern "C"
