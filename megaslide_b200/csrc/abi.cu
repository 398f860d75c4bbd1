// extern "C" entry points of libmegaslide_b200.so: argument validation and kernel dispatch.
// Declarations and the reference interface each one replaces: include/megaslide_b200.h.

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "dsa_attn.cuh"
#include "megaslide_b200.h"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MSL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t elem_size(int dtype) { return dtype == MSL_DTYPE_BF16 ? 2 : 4; }

// Dynamic shared memory the tensor-core kernels may use (the device's opt-in maximum per block).
int tc_smem_limit() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
  return v - 1024;
}

// Validates the geometry and fills the scalar part of AttnParams.
int fill_geometry(const msl_dsa_geometry* g, msl::AttnParams& P) {
  if (!g) return fail(MSL_ERR_INVALID, "geometry is NULL");
  if (g->batch < 1 || g->frames < 1 || g->height < 1 || g->width < 1 || g->heads < 1 || g->head_dim < 1)
    return fail(MSL_ERR_INVALID, "batch/frames/height/width/heads/head_dim must be >= 1");
  if (g->kt < 1 || g->kh < 1 || g->kw < 1 || g->kt % 2 == 0 || g->kh % 2 == 0 || g->kw % 2 == 0)
    return fail(MSL_ERR_INVALID, "kernel_size (%d,%d,%d) must be odd and >= 1 (padding k//2 keeps the size only for odd k)",
                g->kt, g->kh, g->kw);
  if (g->extra < 0) return fail(MSL_ERR_INVALID, "extra must be >= 0");
  if (g->dtype != MSL_DTYPE_F32 && g->dtype != MSL_DTYPE_BF16) return fail(MSL_ERR_INVALID, "unknown dtype %d", g->dtype);
  if (g->q_frame0 < 0 || g->q_frames < 1 || g->q_frame0 + g->q_frames > g->frames)
    return fail(MSL_ERR_INVALID, "query frames [%d, %d) outside [0, %d)", g->q_frame0, g->q_frame0 + g->q_frames, g->frames);
  if (g->kv_frame0 < 0 || g->kv_frames < 1 || g->kv_frame0 + g->kv_frames > g->frames)
    return fail(MSL_ERR_INVALID, "kv frames [%d, %d) outside [0, %d)", g->kv_frame0, g->kv_frame0 + g->kv_frames, g->frames);
  if (!(g->dropout_p >= 0.f && g->dropout_p < 1.f)) return fail(MSL_ERR_INVALID, "dropout_p must be in [0, 1)");
  if (!(g->softmax_scale == g->softmax_scale) || !(g->offset_scale == g->offset_scale))
    return fail(MSL_ERR_INVALID, "softmax_scale / offset_scale is NaN");
  const long long K = static_cast<long long>(g->kt) * g->kh * g->kw;
  if (K > (1 << 20)) return fail(MSL_ERR_UNSUPPORTED, "window too large");
  P = msl::AttnParams{};
  P.B = g->batch; P.T = g->frames; P.H = g->height; P.W = g->width;
  P.nh = g->heads; P.d = g->head_dim; P.kt = g->kt; P.kh = g->kh; P.kw = g->kw;
  P.K = static_cast<int>(K); P.G = g->extra;
  P.q_frame0 = g->q_frame0; P.q_frames = g->q_frames; P.kv_frame0 = g->kv_frame0; P.kv_frames = g->kv_frames;
  P.HW = g->height * g->width;
  P.Nq = static_cast<long long>(g->q_frames) * P.HW;
  P.Nkv = static_cast<long long>(g->kv_frames) * P.HW;
  P.dtype = g->dtype;
  P.scale = g->softmax_scale;
  P.scale_log2 = g->softmax_scale * 1.4426950408889634f;
  P.oscale = g->offset_scale;
  if (g->dropout_p > 0.f) {
    const double th = static_cast<double>(g->dropout_p) * 4294967296.0;
    P.drop_thresh = th >= 4294967295.0 ? 0xffffffffu : static_cast<uint32_t>(th);
    if (P.drop_thresh == 0) P.drop_thresh = 1;
    P.drop_keep_scale = 1.f / (1.f - g->dropout_p);
  } else {
    P.drop_thresh = 0;
    P.drop_keep_scale = 1.f;
  }
  P.seed = g->dropout_seed;
  if (g->algo != MSL_ALGO_AUTO && g->algo != MSL_ALGO_SIMT && g->algo != MSL_ALGO_TC)
    return fail(MSL_ERR_INVALID, "unknown algo %d", g->algo);
  const long long items = static_cast<long long>(P.B) * P.nh * P.Nq;
  if ((items + 7) / 8 > 0x7fffffffLL) return fail(MSL_ERR_UNSUPPORTED, "too many (query, head) items for one launch");
  return MSL_OK;
}

// Chooses 16-byte chunking when every row operand allows it.
int choose_chunking(const msl::AttnParams& P, std::initializer_list<std::pair<const void*, long long>> rows,
                    int* vec, int* maxc) {
  if (!msl::attn_chunking(P.dtype, P.d, vec, maxc))
    return fail(MSL_ERR_UNSUPPORTED, "head_dim %d not supported for dtype %d (max 128)", P.d, P.dtype);
  if (*vec > 1) {
    const size_t es = elem_size(P.dtype);
    bool ok = (static_cast<size_t>(P.d) * es) % 16 == 0;
    for (const auto& r : rows)
      if (r.first && (!aligned16(r.first) || (static_cast<size_t>(r.second) * es) % 16 != 0)) ok = false;
    if (!ok) {
      *vec = 1;
      *maxc = (P.d + 3) / 4;
      if (*maxc > 8) return fail(MSL_ERR_UNSUPPORTED, "unaligned operands with head_dim %d > 32", P.d);
    }
  }
  return MSL_OK;
}

struct BwdWorkspace {
  size_t dk, dv, xds, xp, total;
};

BwdWorkspace bwd_layout(const msl::AttnParams& P, bool accumulate) {
  BwdWorkspace w{};
  const size_t C = static_cast<size_t>(P.nh) * P.d;
  size_t off = 0;
  if (!accumulate) {
    w.dk = off; off = align_up(off + sizeof(float) * P.B * P.Nkv * C, 256);
    w.dv = off; off = align_up(off + sizeof(float) * P.B * P.Nkv * C, 256);
  }
  if (P.G > 0) {
    const size_t n = static_cast<size_t>(P.B) * P.nh * P.Nq * P.G;
    w.xds = off; off = align_up(off + sizeof(float) * n, 256);
    w.xp = off; off = align_up(off + sizeof(float) * n, 256);
  }
  w.total = off;
  return w;
}

int fill_conv(const msl_dwconv_geometry* g, msl::ConvParams& P) {
  if (!g) return fail(MSL_ERR_INVALID, "geometry is NULL");
  if (g->batch < 1 || g->frames < 1 || g->height < 1 || g->width < 1 || g->channels < 1)
    return fail(MSL_ERR_INVALID, "batch/frames/height/width/channels must be >= 1");
  if (g->kt < 1 || g->kh < 1 || g->kw < 1 || g->kt % 2 == 0 || g->kh % 2 == 0 || g->kw % 2 == 0)
    return fail(MSL_ERR_INVALID, "conv kernel (%d,%d,%d) must be odd", g->kt, g->kh, g->kw);
  if (g->dtype != MSL_DTYPE_F32 && g->dtype != MSL_DTYPE_BF16) return fail(MSL_ERR_INVALID, "unknown dtype %d", g->dtype);
  if (g->in_frame0 < 0 || g->in_frames < 1 || g->in_frame0 + g->in_frames > g->frames ||
      g->out_frame0 < 0 || g->out_frames < 1 || g->out_frame0 + g->out_frames > g->frames)
    return fail(MSL_ERR_INVALID, "frame windows outside the volume");
  if (g->zero_outside != 0 && g->zero_outside != 1) return fail(MSL_ERR_INVALID, "zero_outside must be 0 or 1");
  // every tap of every produced frame must be in the input window or outside the volume
  const int pt = g->kt / 2;
  const int need0 = g->out_frame0 - pt < 0 ? 0 : g->out_frame0 - pt;
  const int need1 = g->out_frame0 + g->out_frames + pt > g->frames ? g->frames : g->out_frame0 + g->out_frames + pt;
  if (!g->zero_outside && (need0 < g->in_frame0 || need1 > g->in_frame0 + g->in_frames))
    return fail(MSL_ERR_INVALID, "input frames [%d, %d) do not cover the taps of output frames [%d, %d) (need [%d, %d))",
                g->in_frame0, g->in_frame0 + g->in_frames, g->out_frame0, g->out_frame0 + g->out_frames, need0, need1);
  P.B = g->batch; P.T = g->frames; P.H = g->height; P.W = g->width; P.C = g->channels;
  P.kt = g->kt; P.kh = g->kh; P.kw = g->kw;
  P.in_frame0 = g->in_frame0; P.in_frames = g->in_frames; P.out_frame0 = g->out_frame0; P.out_frames = g->out_frames;
  P.dtype = g->dtype;
  P.HW = g->height * g->width;
  return MSL_OK;
}

}  // namespace

namespace msl {
// Records an error for msl_last_error() from another translation unit of the library.
int record_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace msl

extern "C" {

int32_t msl_abi_version(void) { return MSL_ABI_VERSION; }

uint64_t msl_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* msl_last_error(void) { return g_last_error.c_str(); }

int msl_dsa_attn_fwd(const msl_dsa_geometry* geom, const msl_dsa_fwd_io* io, void* stream) {
  msl::AttnParams P;
  int rc = fill_geometry(geom, P);
  if (rc) return rc;
  if (!io) return fail(MSL_ERR_INVALID, "io is NULL");
  const long long C = static_cast<long long>(P.nh) * P.d;
  if (!io->q || !io->k || !io->v || !io->offsets || !io->out || !io->lse)
    return fail(MSL_ERR_INVALID, "q, k, v, offsets, out and lse are required");
  if (P.G > 0 && (!io->ek || !io->ev)) return fail(MSL_ERR_INVALID, "extra > 0 needs ek and ev");
  if (io->q_ld < C || io->k_ld < C || io->v_ld < C || io->out_ld < C || (P.G > 0 && io->e_ld < C))
    return fail(MSL_ERR_INVALID, "row strides must be >= heads*head_dim = %lld", C);
  if (io->off_ld < static_cast<long long>(P.nh) * P.K * 3)
    return fail(MSL_ERR_INVALID, "off_ld must be >= heads*kt*kh*kw*3");
  P.q = io->q; P.q_ld = io->q_ld; P.k = io->k; P.k_ld = io->k_ld; P.v = io->v; P.v_ld = io->v_ld;
  P.offsets = io->offsets; P.off_ld = io->off_ld;
  P.ek = io->ek; P.ev = io->ev; P.e_ld = io->e_ld;
  P.out = io->out; P.out_ld = io->out_ld; P.lse = io->lse; P.status = io->status; P.probs = io->probs;
  P.saved = io->saved;
  P.off_bias = io->offset_bias;
  if (io->saved && !aligned16(io->saved)) return fail(MSL_ERR_INVALID, "saved must be 16-byte aligned");
  if (geom->algo != MSL_ALGO_SIMT) {
    bool ok = msl::tc_supported(P);
    for (const auto& r : {std::make_pair(io->q, io->q_ld), std::make_pair(io->k, io->k_ld), std::make_pair(io->v, io->v_ld),
                          std::make_pair(static_cast<const void*>(io->out), io->out_ld),
                          std::make_pair(P.G > 0 ? io->ek : nullptr, io->e_ld),
                          std::make_pair(P.G > 0 ? io->ev : nullptr, io->e_ld)})
      if (r.first && (!aligned16(r.first) || r.second % 8 != 0)) ok = false;
    msl::TcLaunch L{};
    if (ok) ok = msl::tc_plan(P, L, tc_smem_limit());
    if (ok) {
      cudaError_t e = msl::launch_attn_fwd_tc(P, L, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "dsa_fwd_tc_kernel launch");
      g_launches.fetch_add(1, std::memory_order_relaxed);
      return MSL_OK;
    }
    if (geom->algo == MSL_ALGO_TC || io->probs || io->saved)
      return fail(MSL_ERR_UNSUPPORTED, "tensor-core path (%s) needs bf16, head_dim %% 8 == 0 in [16,128], 16-byte aligned rows",
                  (io->probs || io->saved) ? "required by the probs / saved outputs" : "algo = MSL_ALGO_TC");
  }
  if (io->probs || io->saved)
    return fail(MSL_ERR_UNSUPPORTED, "the probs / saved outputs are written by the tensor-core path only (algo != SIMT)");
  int vec = 1, maxc = 1;
  rc = choose_chunking(P, {{io->q, io->q_ld}, {io->k, io->k_ld}, {io->v, io->v_ld}, {io->out, io->out_ld},
                           {P.G > 0 ? io->ek : nullptr, io->e_ld}, {P.G > 0 ? io->ev : nullptr, io->e_ld}},
                       &vec, &maxc);
  if (rc) return rc;
  cudaError_t e = msl::launch_attn_fwd(P, vec, maxc, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dsa_fwd_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSL_OK;
}

size_t msl_dsa_saved_bytes(const msl_dsa_geometry* geom) {
  msl::AttnParams P;
  if (fill_geometry(geom, P)) return 0;
  return static_cast<size_t>(msl::saved_bytes(P));
}

size_t msl_dsa_attn_bwd_workspace_bytes(const msl_dsa_geometry* geom, int32_t accumulate_mode) {
  msl::AttnParams P;
  if (fill_geometry(geom, P)) return 0;
  return bwd_layout(P, accumulate_mode != 0).total;
}

int msl_dsa_attn_bwd(const msl_dsa_geometry* geom, const msl_dsa_bwd_io* io, void* workspace,
                     size_t workspace_bytes, void* stream) {
  msl::AttnParams P;
  int rc = fill_geometry(geom, P);
  if (rc) return rc;
  if (!io) return fail(MSL_ERR_INVALID, "io is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long C = static_cast<long long>(P.nh) * P.d;
  if (!io->q || !io->k || !io->v || !io->offsets || !io->out || !io->lse || !io->dout || !io->dq || !io->doffsets)
    return fail(MSL_ERR_INVALID, "q, k, v, offsets, out, lse, dout, dq and doffsets are required");
  const bool accumulate = io->dk_acc != nullptr;
  if (accumulate) {
    if (!io->dv_acc) return fail(MSL_ERR_INVALID, "dk_acc given without dv_acc");
    if (io->acc_ld < C) return fail(MSL_ERR_INVALID, "acc_ld must be >= %lld", C);
  } else {
    if (!io->dk || !io->dv) return fail(MSL_ERR_INVALID, "dk and dv (or dk_acc and dv_acc) are required");
    if (io->dkv_ld < C) return fail(MSL_ERR_INVALID, "dkv_ld must be >= %lld", C);
  }
  if (P.G > 0 && (!io->ek || !io->ev || !io->dek || !io->dev))
    return fail(MSL_ERR_INVALID, "extra > 0 needs ek, ev, dek and dev");
  if (io->q_ld < C || io->k_ld < C || io->v_ld < C || io->out_ld < C || io->dout_ld < C || io->dq_ld < C ||
      (P.G > 0 && io->e_ld < C))
    return fail(MSL_ERR_INVALID, "row strides must be >= heads*head_dim = %lld", C);
  if (io->off_ld < static_cast<long long>(P.nh) * P.K * 3 || io->doff_ld < static_cast<long long>(P.nh) * P.K * 3)
    return fail(MSL_ERR_INVALID, "off_ld / doff_ld must be >= heads*kt*kh*kw*3");
  const BwdWorkspace L = bwd_layout(P, accumulate);
  if (L.total > 0) {
    if (!workspace || workspace_bytes < L.total)
      return fail(MSL_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", L.total, workspace ? workspace_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return fail(MSL_ERR_INVALID, "workspace must be 256-byte aligned");
  }
  char* ws = static_cast<char*>(workspace);
  P.q = io->q; P.q_ld = io->q_ld; P.k = io->k; P.k_ld = io->k_ld; P.v = io->v; P.v_ld = io->v_ld;
  P.offsets = io->offsets; P.off_ld = io->off_ld;
  P.ek = io->ek; P.ev = io->ev; P.e_ld = io->e_ld;
  P.out = const_cast<void*>(io->out); P.out_ld = io->out_ld; P.lse = const_cast<float*>(io->lse);
  P.dout = io->dout; P.dout_ld = io->dout_ld; P.dq = io->dq; P.dq_ld = io->dq_ld;
  if (io->doff_dtype != MSL_DTYPE_F32 && io->doff_dtype != MSL_DTYPE_BF16)
    return fail(MSL_ERR_INVALID, "unknown doff_dtype %d", io->doff_dtype);
  P.doffsets = io->doffsets; P.doff_ld = io->doff_ld; P.doff_bf16 = io->doff_dtype == MSL_DTYPE_BF16;
  P.status = io->status;
  P.probs = const_cast<float*>(io->probs);
  P.saved = const_cast<void*>(io->saved);
  P.off_bias = io->offset_bias;
  if (io->saved && !aligned16(io->saved)) return fail(MSL_ERR_INVALID, "saved must be 16-byte aligned");
  if (accumulate) {
    P.dk_acc = io->dk_acc; P.dv_acc = io->dv_acc; P.acc_ld = io->acc_ld;
  } else {
    P.dk_acc = reinterpret_cast<float*>(ws + L.dk);
    P.dv_acc = reinterpret_cast<float*>(ws + L.dv);
    P.acc_ld = C;
  }
  if (P.G > 0) {
    P.extra_ds = reinterpret_cast<float*>(ws + L.xds);
    P.extra_p = reinterpret_cast<float*>(ws + L.xp);
    P.dek = io->dek; P.dev = io->dev;
  }
  // tensor-core backward: bf16, softmax weights saved by the forward, aligned rows
  msl::TcLaunch TL{};
  bool use_tc = false;
  if (geom->algo != MSL_ALGO_SIMT && P.probs && P.saved) {
    use_tc = msl::tc_bwd_supported(P);
    for (const auto& r : {std::make_pair(io->q, io->q_ld), std::make_pair(io->k, io->k_ld), std::make_pair(io->v, io->v_ld),
                          std::make_pair(io->out, io->out_ld), std::make_pair(io->dout, io->dout_ld),
                          std::make_pair(static_cast<const void*>(io->dq), io->dq_ld)})
      if (!aligned16(r.first) || r.second % 8 != 0) use_tc = false;
    if (!aligned16(P.dk_acc) || !aligned16(P.dv_acc) || P.acc_ld % 4 != 0) use_tc = false;
    if (use_tc) use_tc = msl::tc_bwd_plan(P, TL, tc_smem_limit());
  }
  if (geom->algo == MSL_ALGO_TC && !use_tc)
    return fail(MSL_ERR_UNSUPPORTED, "tensor-core backward needs probs and saved from the tensor-core forward, bf16, "
                                     "at most one key-buffer chunk of extra keys, head_dim %% 8 == 0 in [16,128] and "
                                     "16-byte aligned rows");
  int vec = 1, maxc = 1;
  rc = choose_chunking(P, {{io->q, io->q_ld}, {io->k, io->k_ld}, {io->v, io->v_ld}, {io->out, io->out_ld},
                           {io->dout, io->dout_ld}, {io->dq, io->dq_ld},
                           {P.G > 0 ? io->ek : nullptr, io->e_ld}, {P.G > 0 ? io->ev : nullptr, io->e_ld}},
                       &vec, &maxc);
  if (rc) return rc;
  if (vec > 1) {
    // float32 accumulator rows take 16-byte vector atomics
    if (!aligned16(P.dk_acc) || !aligned16(P.dv_acc) || (P.acc_ld % 4) != 0) {
      vec = 1;
      maxc = (P.d + 3) / 4;
      if (maxc > 8) return fail(MSL_ERR_UNSUPPORTED, "unaligned accumulators with head_dim %d > 32", P.d);
    }
  }
  cudaError_t e;
  if (!accumulate) {
    e = cudaMemsetAsync(ws + L.dk, 0, L.dv - L.dk, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(ws + L.dv, 0, sizeof(float) * P.B * P.Nkv * C, s);
    if (e != cudaSuccess) return cuda_fail(e, "clearing dK/dV accumulators");
  }
  if (P.G > 0) {
    const size_t nb = sizeof(float) * P.B * P.G * C;
    e = cudaMemsetAsync(P.dek, 0, nb, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(P.dev, 0, nb, s);
    if (e != cudaSuccess) return cuda_fail(e, "clearing dek/dev");
  }
  if (use_tc) {
    e = msl::launch_attn_bwd_tc(P, TL, s);  // the tensor-core kernel, then its CUDA-core fallback tiles
    if (e != cudaSuccess) return cuda_fail(e, "dsa_bwd_tc_kernel launch");
    g_launches.fetch_add(2, std::memory_order_relaxed);
  } else {
    e = msl::launch_attn_bwd(P, vec, maxc, s);
    if (e != cudaSuccess) return cuda_fail(e, "dsa_bwd_kernel launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  if (P.G > 0) {
    e = msl::launch_attn_extra_grad(P, s);
    if (e != cudaSuccess) return cuda_fail(e, "dsa_extra_grad_kernel launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  if (!accumulate) {
    const long long rows = static_cast<long long>(P.B) * P.Nkv;
    e = msl::launch_convert_f32(P.dk_acc, C, io->dk, io->dkv_ld, P.dtype, rows, C, s);
    if (e == cudaSuccess) e = msl::launch_convert_f32(P.dv_acc, C, io->dv, io->dkv_ld, P.dtype, rows, C, s);
    if (e != cudaSuccess) return cuda_fail(e, "convert_f32_kernel launch");
    g_launches.fetch_add(2, std::memory_order_relaxed);
  }
  return MSL_OK;
}

int msl_dwconv3d_fwd(const msl_dwconv_geometry* geom, const void* x, int64_t x_ld, const float* weight,
                     const float* bias, const float* bias2, int32_t epilogue, const void* aux, int64_t aux_ld,
                     void* y, int64_t y_ld, int32_t y_dtype, void* stream) {
  msl::ConvParams P;
  int rc = fill_conv(geom, P);
  if (rc) return rc;
  if (!x || !weight || !y) return fail(MSL_ERR_INVALID, "x, weight and y are required");
  if (epilogue != MSL_EPI_NONE && epilogue != MSL_EPI_GELU && epilogue != MSL_EPI_GELU_GRAD &&
      epilogue != MSL_EPI_ACCUM)
    return fail(MSL_ERR_INVALID, "unknown epilogue %d", epilogue);
  if (epilogue == MSL_EPI_ACCUM && y_dtype != MSL_DTYPE_F32) return fail(MSL_ERR_INVALID, "ACCUM needs a float32 y");
  if (epilogue == MSL_EPI_GELU_GRAD && (!aux || aux_ld < P.C)) return fail(MSL_ERR_INVALID, "GELU_GRAD needs aux rows");
  if (x_ld < P.C || y_ld < P.C) return fail(MSL_ERR_INVALID, "row strides must be >= channels");
  if (y_dtype != MSL_DTYPE_F32 && y_dtype != MSL_DTYPE_BF16) return fail(MSL_ERR_INVALID, "unknown y_dtype %d", y_dtype);
  cudaError_t e = msl::launch_dwconv_fwd(P, x, x_ld, weight, bias, bias2, epilogue, aux, aux_ld, y, y_ld, y_dtype,
                                         false, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwconv_fwd_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSL_OK;
}

int msl_dwconv3d_bwd_data(const msl_dwconv_geometry* geom, const void* dy, int64_t dy_ld, const float* weight,
                          void* dx, int64_t dx_ld, void* stream) {
  msl::ConvParams P;
  int rc = fill_conv(geom, P);
  if (rc) return rc;
  if (!dy || !weight || !dx) return fail(MSL_ERR_INVALID, "dy, weight and dx are required");
  if (dy_ld < P.C || dx_ld < P.C) return fail(MSL_ERR_INVALID, "row strides must be >= channels");
  cudaError_t e = msl::launch_dwconv_fwd(P, dy, dy_ld, weight, nullptr, nullptr, MSL_EPI_NONE, nullptr, 0, dx, dx_ld,
                                         P.dtype, true, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwconv_fwd_kernel(transposed) launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSL_OK;
}

int msl_dwconv3d_bwd_data_acc(const msl_dwconv_geometry* geom, const void* dy, int64_t dy_ld, const float* weight,
                              float* dx, int64_t dx_ld, void* stream) {
  msl::ConvParams P;
  int rc = fill_conv(geom, P);
  if (rc) return rc;
  if (!dy || !weight || !dx) return fail(MSL_ERR_INVALID, "dy, weight and dx are required");
  if (dy_ld < P.C || dx_ld < P.C) return fail(MSL_ERR_INVALID, "row strides must be >= channels");
  cudaError_t e = msl::launch_dwconv_fwd(P, dy, dy_ld, weight, nullptr, nullptr, MSL_EPI_ACCUM, nullptr, 0, dx, dx_ld,
                                         MSL_DTYPE_F32, true, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwconv_fwd_kernel(transposed, accumulate) launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSL_OK;
}

int msl_dwconv3d_bwd_weight(const msl_dwconv_geometry* geom, const void* dy, int64_t dy_ld, int32_t dy_dtype,
                            const void* x, int64_t x_ld, float* dweight, float* dbias, void* stream) {
  msl::ConvParams P;
  int rc = fill_conv(geom, P);
  if (rc) return rc;
  if (!dy || !x || !dweight) return fail(MSL_ERR_INVALID, "dy, x and dweight are required");
  if (dy_ld < P.C || x_ld < P.C) return fail(MSL_ERR_INVALID, "row strides must be >= channels");
  if (dy_dtype != MSL_DTYPE_F32 && dy_dtype != MSL_DTYPE_BF16) return fail(MSL_ERR_INVALID, "unknown dy_dtype %d", dy_dtype);
  cudaError_t e = msl::launch_dwconv_wgrad(P, dy, dy_ld, dy_dtype, x, x_ld, dweight, dbias,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwconv_wgrad_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSL_OK;
}

int msl_offsets_absmax(const float* offsets, int64_t rows, int64_t ld, const float* bias, int32_t heads, int32_t taps,
                       float offset_scale, float* out3, void* stream) {
  if (!offsets || !out3) return fail(MSL_ERR_INVALID, "offsets and out3 are required");
  if (rows < 0 || heads < 1 || taps < 1 || ld < static_cast<int64_t>(heads) * taps * 3)
    return fail(MSL_ERR_INVALID, "bad offsets shape");
  if (rows == 0) return MSL_OK;
  cudaError_t e = msl::launch_offsets_absmax(offsets, rows, ld, bias, heads, taps, offset_scale, out3,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "offsets_absmax_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSL_OK;
}

int msl_convert_f32(const float* src, int64_t src_ld, void* dst, int64_t dst_ld, int32_t dtype, int64_t rows,
                    int64_t cols, void* stream) {
  if (!src || !dst) return fail(MSL_ERR_INVALID, "src and dst are required");
  if (dtype != MSL_DTYPE_F32 && dtype != MSL_DTYPE_BF16) return fail(MSL_ERR_INVALID, "unknown dtype %d", dtype);
  if (rows < 0 || cols < 0 || src_ld < cols || dst_ld < cols) return fail(MSL_ERR_INVALID, "bad matrix shape");
  if (rows == 0 || cols == 0) return MSL_OK;
  cudaError_t e = msl::launch_convert_f32(src, src_ld, dst, dst_ld, dtype, rows, cols, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "convert_f32_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSL_OK;
}

}  // extern "C"
