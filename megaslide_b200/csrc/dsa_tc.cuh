// Building blocks shared by the tensor-core ("key envelope") kernels of the deformable gather
// attention (forward: dsa_tc.cu, backward: dsa_tc_bwd.cu).  Both kernels run 512 threads per CTA on
// a tile of queries of one frame, one head and one sample, walk the tile's key envelope one frame
// ("plane") at a time in chunks of at most `maxkeys` keys, and do the dense per-chunk products with
// mma.sync (bf16 in, fp32 accumulate) on operands in shared memory.  Key / value chunks arrive by TMA
// tensor copies (one 8-key box per chunk row segment, completing on an mbarrier) when the K / V
// buffers meet TMA's alignment rules, else by cp.async.
#pragma once

#include <cuda.h>

#include <math.h>
#include <stdint.h>

#include "dsa_attn.cuh"
#include "dsa_simt.cuh"
#include "msl_common.cuh"

namespace msl {
namespace tc {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kTileW = 8;               // tile columns; a 16-query row group = 2 tile rows
constexpr int kEnvWords = 16 + 3 * 96;  // envelope ints + base-grid tables of the tile (<= 96 each)
// Dense P~ matrices are accumulated with 32-bit integer shared-memory atomics in fixed point:
// value * 2^24.  Entries are sums of trilinear weights (<= 1) times softmax weights whose sum is at
// most the dropout keep scale 1/(1-p), so they stay below 2^32 for p <= 0.9 (host-checked).
constexpr float kPtScale = 16777216.f;
constexpr float kPtInv = 1.f / 16777216.f;

// ------------------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3},{%4,%5,%6,%7},{%8,%9},{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma1688(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3},{%4,%5},{%6},{%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g));
}
__device__ __forceinline__ void cp_async8(uint32_t saddr, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(saddr), "l"(g));
}
__device__ __forceinline__ void cp_async4(uint32_t saddr, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(saddr), "l"(g));
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// orders this thread's earlier generic-proxy shared-memory accesses before its later TMA writes
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// 5-d tiled tensor copy global -> this CTA's shared memory, completing on mbarrier `bar` (no multicast)
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], "
      "[%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
      : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------ tile geometry
struct TileCtx {
  int b, head, tl, tg, qh0, qw0;
};

// tile index -> (sample, tile row, tile column, local frame, head).  Heads vary fastest, then frames:
// the CTAs that run together are the heads and neighbouring frames of one spatial tile, whose key
// envelopes overlap (samples reach several frames away), so their K/V chunk reads and dK/dV
// accumulator adds meet in L2 instead of being spread over the whole launch.
__device__ __forceinline__ TileCtx decode_tile_index(const AttnParams& P, const TcLaunch& L, int tile_h, long long t) {
  TileCtx c;
  c.head = static_cast<int>(t % P.nh);
  t /= P.nh;
  c.tl = static_cast<int>(t % P.q_frames);
  t /= P.q_frames;
  const int iw = static_cast<int>(t % L.tiles_w);
  t /= L.tiles_w;
  const int ih = static_cast<int>(t % L.tiles_h);
  c.b = static_cast<int>(t / L.tiles_h);
  c.tg = P.q_frame0 + c.tl;
  c.qh0 = ih * tile_h;
  c.qw0 = iw * kTileW;
  return c;
}
// the CTA's tile (one CTA per tile)
__device__ __forceinline__ TileCtx decode_tile(const AttnParams& P, const TcLaunch& L, int tile_h) {
  return decode_tile_index(P, L, tile_h, blockIdx.x);
}

// query c (0..15) of row group r: tile rows 2r, 2r+1
__device__ __forceinline__ void query_hw(const TileCtx& T, int r, int c, int& qh, int& qw) {
  qh = T.qh0 + 2 * r + (c >> 3);
  qw = T.qw0 + (c & 7);
}

// Chunking of an envelope axis [lo, hi] into windows of `len` with one element of overlap.
__device__ __forceinline__ int axis_chunks(int lo, int hi, int len) {
  const int n = hi - lo + 1;
  if (n <= len) return 1;
  return 1 + (n - len + (len - 2)) / (len - 1);
}
__device__ __forceinline__ int axis_chunk_of(int v, int lo, int len, int nchunks) {
  if (nchunks == 1) return 0;
  const int i = (v - lo) / (len - 1);
  return i < nchunks - 1 ? i : nchunks - 1;
}

struct Env {
  int zlo, zhi, ylo, yhi, xlo, xhi;
  int cw, R, ny, nx;  // column-chunk width, rows per chunk, chunk counts
  int kst;            // key row stride in a chunk: cw rounded up to 8 (chunk key = (y - ya) * kst + x - xa)
  int pg;             // planes per chunk (1, or 2 when two planes' keys fit one chunk)
  int kpp;            // key offset of a chunk's second plane (multiple of 16; pg == 2)
};

// Chunk shape for an envelope [ylo, yhi] x [xlo, xhi] and `maxkeys` keys per chunk: columns split into
// windows of at most min(maxkeys / 2, 32), rows into windows of maxkeys / kst (>= 2, as maxkeys % 16 == 0).
__device__ __forceinline__ void chunk_shape(Env& E, int maxkeys) {
  const int nxk = E.xhi - E.xlo + 1;
  E.cw = min(nxk, min(maxkeys / 2, 32));  // at most 32 columns: one TMA box per chunk row
  E.kst = (E.cw + 7) & ~7;
  E.R = maxkeys / E.kst;
  E.ny = axis_chunks(E.ylo, E.yhi, E.R);
  E.nx = axis_chunks(E.xlo, E.xhi, E.cw);
  E.pg = 1;
  E.kpp = 0;
}

// Two planes per chunk when one chunk holds a whole plane and two planes' keys (each padded to whole
// 16-key tiles) fit `maxkeys`: a sample whose two trilinear planes share the chunk is visited once.
__device__ __forceinline__ void chunk_pair_planes(Env& E, int maxkeys) {
  const int kp = ((E.yhi - E.ylo + 1) * E.kst + 15) & ~15;
  if (E.ny == 1 && E.nx == 1 && E.zhi > E.zlo && 2 * kp <= maxkeys) {
    E.pg = 2;
    E.kpp = kp;
  }
}

// Base-grid values 2a/max(S-1,1) - 1 of the window positions a tile can reach, per axis, computed once
// per CTA with the same float32 operations as base_grid(); tz covers frames tg - kt/2 .. tg + kt/2,
// ty rows qh0 - kh/2 .. qh0 + tile_h - 1 + kh/2, tx columns qw0 - kw/2 .. qw0 + 7 + kw/2.
struct Tabs {
  const float *tz, *ty, *tx;
};

__device__ __forceinline__ void fill_tabs(const AttnParams& P, const TileCtx& T, int tile_h, float* tz, float* ty,
                                          float* tx) {
  for (int i = threadIdx.x; i < P.kt + P.kh + tile_h - 1 + P.kw + kTileW - 1; i += kThreads) {
    if (i < P.kt) {
      tz[i] = base_grid(T.tg + i - P.kt / 2, P.T);
    } else if (i < P.kt + P.kh + tile_h - 1) {
      const int k = i - P.kt;
      ty[k] = base_grid(T.qh0 + k - P.kh / 2, P.H);
    } else {
      const int k = i - P.kt - P.kh - tile_h + 1;
      tx[k] = base_grid(T.qw0 + k - P.kw / 2, P.W);
    }
  }
}

// sample_coords() with the base grid read from the tables: (qy, qx) are the query's row / column
// inside the tile, (it, ih, iw) the window index.  Same float32 operations, same result.
__device__ __forceinline__ void tab_coords(const AttnParams& P, const Tabs& tb, int qy, int qx, int it, int ih, int iw,
                                           float o0, float o1, float o2, float& pt, float& ph, float& pw) {
  float gx = tb.tx[qx + iw], gy = tb.ty[qy + ih], gz = tb.tz[it];
  if (P.T > 1) gx = __fadd_rn(gx, __fdiv_rn(__fmul_rn(o0, P.oscale), static_cast<float>(P.T - 1)));
  if (P.H > 1) gy = __fadd_rn(gy, __fdiv_rn(__fmul_rn(o1, P.oscale), static_cast<float>(P.H - 1)));
  if (P.W > 1) gz = __fadd_rn(gz, __fdiv_rn(__fmul_rn(o2, P.oscale), static_cast<float>(P.W - 1)));
  pw = unnormalize_clip(gx, P.W);
  ph = unnormalize_clip(gy, P.H);
  pt = unnormalize_clip(gz, P.T);
}

// Window index (it, ih, iw) of sample j, advanced by `step` samples without integer division.
struct WinIdx {
  int it, ih, iw;
  __device__ __forceinline__ void init(int j, int kh, int kw) {
    it = j / (kh * kw);
    const int r = j - it * kh * kw;
    ih = r / kw;
    iw = r - ih * kw;
  }
  __device__ __forceinline__ void advance(int step, int kh, int kw) {
    iw += step;
    while (iw >= kw) {
      iw -= kw;
      if (++ih == kh) {
        ih = 0;
        ++it;
      }
    }
  }
};

// ------------------------------------------------------------------------------ sample records
// Packed per-sample record (0 = inactive sample):
//   bits  0-11, 12-23, 24-35: fractions pt - t0, ph - h0, pw - w0 as 12-bit unorm
//   bits 36-40: t0 - zlo + 1,  41-48: h0 - ylo,  49-56: w0 - xlo,  bit 63: active
//   bits 57-62: free for kernel-specific flags
__device__ __forceinline__ uint32_t quant12(float f) {
  int u = __float2int_rn(f * 4096.f);
  return static_cast<uint32_t>(u < 0 ? 0 : (u > 4095 ? 4095 : u));
}
__device__ __forceinline__ unsigned long long pack_rec(float ft, float fh, float fw, int dz, int dy, int dx) {
  return static_cast<unsigned long long>(quant12(ft)) | (static_cast<unsigned long long>(quant12(fh)) << 12) |
         (static_cast<unsigned long long>(quant12(fw)) << 24) | (static_cast<unsigned long long>(dz) << 36) |
         (static_cast<unsigned long long>(dy) << 41) | (static_cast<unsigned long long>(dx) << 49) | (1ull << 63);
}
struct Rec {
  float ft, fh, fw;
  int t0, h0, w0;
};
__device__ __forceinline__ Rec unpack_rec(unsigned long long v, const Env& E) {
  Rec r;
  r.ft = static_cast<float>(v & 0xfffu) * (1.f / 4096.f);
  r.fh = static_cast<float>((v >> 12) & 0xfffu) * (1.f / 4096.f);
  r.fw = static_cast<float>((v >> 24) & 0xfffu) * (1.f / 4096.f);
  r.t0 = E.zlo - 1 + static_cast<int>((v >> 36) & 0x1fu);
  r.h0 = E.ylo + static_cast<int>((v >> 41) & 0xffu);
  r.w0 = E.xlo + static_cast<int>((v >> 49) & 0xffu);
  return r;
}
// true when the active record has a corner in plane zrel (relative frame, zlo -> 1)
__device__ __forceinline__ bool rec_in_plane(unsigned long long v, int zrel) {
  return (v >> 63) && static_cast<unsigned>(zrel - static_cast<int>((v >> 36) & 0x1fu)) <= 1u;
}
// weight factor of the lower (upper = 0) or upper corner along one axis from the fraction
__device__ __forceinline__ float frac_weight(float f, int upper) { return upper ? f : 1.f - f; }

// ------------------------------------------------------------------------------ chunk operands
// Loads keys (z, y, x) for y in [ya, yb], x in [xa, xb] of one head into kbuf rows
// (y - ya) * ncw + (x - xa); rows past the chunk (up to nkp) and keys outside the volume or the
// K/V frame window are zero.  DCH = head_dim / 8 sixteen-byte chunks per key.
template <int DCH>
__device__ __forceinline__ void load_chunk(const AttnParams& P, const TileCtx& T, __nv_bfloat16* kbuf, int rs,
                                           const __nv_bfloat16* base, long long ld, int z, int ya, int yb, int xa,
                                           int xb, int nkp) {
  const int ncw = xb - xa + 1;
  const int nk = (yb - ya + 1) * ncw;
  const int zl = z - P.kv_frame0;
  const bool zok = zl >= 0 && zl < P.kv_frames;
  const __nv_bfloat16* gb = base + static_cast<long long>(T.b) * P.Nkv * ld + T.head * P.d;
  // one key row (ncw keys x DCH chunks) per step; row-major within the chunk
  const int per_row = ncw * DCH;
  for (int y = ya; y <= yb; ++y) {
    const bool yok = zok && y >= 0 && y < P.H;
    const int kb = (y - ya) * ncw;
    const __nv_bfloat16* grow = gb + ((static_cast<long long>(zl) * P.H + y) * P.W) * ld;
    for (int idx = threadIdx.x; idx < per_row; idx += kThreads) {
      const int kx = idx / DCH, ch = idx - (idx / DCH) * DCH;  // DCH is a compile-time constant
      const int x = xa + kx;
      __nv_bfloat16* dst = kbuf + static_cast<size_t>(kb + kx) * rs + ch * 8;
      if (yok && x >= 0 && x < P.W)
        cp_async16(smem_u32(dst), grow + static_cast<long long>(x) * ld + ch * 8);
      else
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  for (int idx = nk * DCH + threadIdx.x; idx < nkp * DCH; idx += kThreads) {  // padding keys
    const int key = idx / DCH, ch = idx - (idx / DCH) * DCH;
    *reinterpret_cast<uint4*>(kbuf + static_cast<size_t>(key) * rs + ch * 8) = make_uint4(0u, 0u, 0u, 0u);
  }
  cp_async_wait_all();
}

// srow[16 queries][nkp keys] = A . kbuf^T for one 16-row group: A in registers (m16n8k16 A fragments
// of the group's rows, DCH / 2 k-steps plus an m16n8k8 tail for odd DCH); the WPG warps of the group
// split the 16-key column blocks round robin (`part` = warp index within the group).
template <int DCH, int WPG>
__device__ __forceinline__ void dense_scores(const __nv_bfloat16* kbuf, int rs, float* srow, int sld, int part, int nkp,
                                             const uint32_t (&qa)[DCH / 2 > 0 ? DCH / 2 : 1][4],
                                             const uint32_t (&qt)[2]) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  for (int gi = part; gi * 16 < nkp; gi += WPG) {
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    // x4 matrices: (keys +0..7, d +0..7) (keys +0..7, d +8..15) (keys +8..15, d +0..7) (keys +8..15, d +8..15)
    const int key = gi * 16 + rr + ((mi >> 1) ? 8 : 0);
    const __nv_bfloat16* rowp = kbuf + static_cast<size_t>(key) * rs + ((mi & 1) ? 8 : 0);
#pragma unroll
    for (int ks = 0; ks < DCH / 2; ++ks) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(rowp + ks * 16), b0, b1, b2, b3);
      mma16816(c0, qa[ks], b0, b1);
      mma16816(c1, qa[ks], b2, b3);
    }
    if constexpr (DCH & 1) {
      const int key2 = gi * 16 + rr + ((mi & 1) ? 8 : 0);
      uint32_t e0, e1;
      ldsm_x2(smem_u32(kbuf + static_cast<size_t>(key2) * rs + (DCH - 1) * 8), e0, e1);
      mma1688(c0, qt[0], qt[1], e0);
      mma1688(c1, qt[0], qt[1], e1);
    }
    float* p0 = srow + static_cast<size_t>(g) * sld + gi * 16 + 2 * t4;
    float* p1 = srow + static_cast<size_t>(g + 8) * sld + gi * 16 + 2 * t4;
    *reinterpret_cast<float2*>(p0) = make_float2(c0[0], c0[1]);
    *reinterpret_cast<float2*>(p1) = make_float2(c0[2], c0[3]);
    *reinterpret_cast<float2*>(p0 + 8) = make_float2(c1[0], c1[1]);
    *reinterpret_cast<float2*>(p1 + 8) = make_float2(c1[2], c1[3]);
  }
}

// o[16][d tiles nt0..nt1) += A[16][nkp] . vbuf[nkp][d] for one 16-row group.  A is read from the
// group's rows of a shared fp32 matrix (FIXED: u32 fixed point, scaled by 2^-24) and rounded to bf16
// fragments; vbuf rows (keys) through ldmatrix.trans.  o[j] accumulates d tile nt0 + j.
template <int DCH, int TPW, bool FIXED>
__device__ __forceinline__ void av_product(const float* arow, int sld, const __nv_bfloat16* vbuf, int rs, int nt0,
                                           int nt1, int nkp, float (&o)[TPW + 1][4]) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  for (int kk = 0; kk * 16 < nkp; ++kk) {
    const float* a0p = arow + static_cast<size_t>(g) * sld + kk * 16 + 2 * t4;
    const float* a1p = arow + static_cast<size_t>(g + 8) * sld + kk * 16 + 2 * t4;
    uint32_t a[4];
    if constexpr (FIXED) {
      const uint2 x0 = *reinterpret_cast<const uint2*>(a0p);
      const uint2 x1 = *reinterpret_cast<const uint2*>(a1p);
      const uint2 x2 = *reinterpret_cast<const uint2*>(a0p + 8);
      const uint2 x3 = *reinterpret_cast<const uint2*>(a1p + 8);
      a[0] = pack_bf16(x0.x * kPtInv, x0.y * kPtInv);
      a[1] = pack_bf16(x1.x * kPtInv, x1.y * kPtInv);
      a[2] = pack_bf16(x2.x * kPtInv, x2.y * kPtInv);
      a[3] = pack_bf16(x3.x * kPtInv, x3.y * kPtInv);
    } else {
      const float2 x0 = *reinterpret_cast<const float2*>(a0p);
      const float2 x1 = *reinterpret_cast<const float2*>(a1p);
      const float2 x2 = *reinterpret_cast<const float2*>(a0p + 8);
      const float2 x3 = *reinterpret_cast<const float2*>(a1p + 8);
      a[0] = pack_bf16(x0.x, x0.y);
      a[1] = pack_bf16(x1.x, x1.y);
      a[2] = pack_bf16(x2.x, x2.y);
      a[3] = pack_bf16(x3.x, x3.y);
    }
    // x4.trans matrices: (keys +0..7, d nt) (keys +8..15, d nt) (keys +0..7, d nt+1) (keys +8..15, d nt+1)
    const int key = kk * 16 + rr + ((mi & 1) ? 8 : 0);
    const __nv_bfloat16* rowp = vbuf + static_cast<size_t>(key) * rs;
#pragma unroll
    for (int jj = 0; jj < TPW; jj += 2) {
      const int nt = nt0 + jj;
      if (nt + 1 < nt1) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(rowp + (nt + (mi >> 1)) * 8), b0, b1, b2, b3);
        mma16816(o[jj], a, b0, b1);
        mma16816(o[jj + 1], a, b2, b3);
      } else if (nt < nt1) {
        uint32_t b0, b1;
        ldsm_x2_t(smem_u32(rowp + nt * 8), b0, b1);
        mma16816(o[jj], a, b0, b1);
      }
    }
  }
}

// ------------------------------------------------------------------------------ masked chunks
// ------------------------------------------------------------------------------ scalar helpers
// float -> nearest int for |v| < 2^22 and back, with one add (no conversion instruction)
__device__ __forceinline__ int fix_round(float v) { return __float_as_int(v + 12582912.f) - 0x4B400000; }
__device__ __forceinline__ float fix_float(int v) { return __int_as_float(v + 0x4B400000) - 12582912.f; }

// position of the o-th (0-based) set bit of m (which has more than o set bits)
__device__ __forceinline__ int nth_bit(uint32_t m, int o) {
  int base = 0;
#pragma unroll
  for (int w = 16; w > 0; w >>= 1) {
    const int c = __popc(m & ((1u << w) - 1u));
    if (o >= c) {
      o -= c;
      m >>= w;
      base += w;
    }
  }
  return base;
}

// record -> corner and fractions (fractions exactly q / 4096, built from the float bit pattern)
__device__ __forceinline__ Rec decode_rec(unsigned long long v, const Env& E) {
  Rec r;
  r.ft = __uint_as_float(0x3F800000u | ((static_cast<uint32_t>(v) & 0xfffu) << 11)) - 1.f;
  r.fh = __uint_as_float(0x3F800000u | ((static_cast<uint32_t>(v >> 12) & 0xfffu) << 11)) - 1.f;
  r.fw = __uint_as_float(0x3F800000u | ((static_cast<uint32_t>(v >> 24) & 0xfffu) << 11)) - 1.f;
  r.t0 = E.zlo - 1 + static_cast<int>((v >> 36) & 0x1fu);
  r.h0 = E.ylo + static_cast<int>((v >> 41) & 0xffu);
  r.w0 = E.xlo + static_cast<int>((v >> 49) & 0xffu);
  return r;
}

// Hit lists are bucketed by (chunk, frame): record bits 61-62 hold the sample's chunk within its planes
// (iy * nx + ix, when tile masks are kept, else 0); bucket = chunk * 32 + (t0 - zlo + 1).  The hits of
// chunk c in plane zr are the buckets c * 32 + zr (upper corner there) and c * 32 + zr + 1 (lower):
// one contiguous range [bstart[c * 32 + zr], bstart[c * 32 + zr + 2]).
// record flags (both kernels; set by the forward, read by the backward): grid coordinate strictly
// inside (0, S-1) along t / h / w, dropout keep
constexpr int kBitInT = 57, kBitInH = 58, kBitInW = 59, kBitKeep = 60;
constexpr int kBitChunk = 61;
constexpr int kBuckets = 128;
__device__ __forceinline__ int rec_bucket(unsigned long long v) {
  return static_cast<int>((v >> kBitChunk) & 3u) * 32 + static_cast<int>((v >> 36) & 0x1fu);
}
// exclusive scan of the kBuckets counts in bcur by warp 0: bucket starts in bstart[0 .. kBuckets], the
// counts become fill cursors
__device__ __forceinline__ void scan_buckets(int* bcur, int* bstart) {
  const int lane = threadIdx.x & 31;
  const int4 c = reinterpret_cast<const int4*>(bcur)[lane];
  const int s = c.x + c.y + c.z + c.w;
  int incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const int e0 = incl - s, e1 = e0 + c.x, e2 = e1 + c.y, e3 = e2 + c.z;
  reinterpret_cast<int4*>(bstart)[lane] = make_int4(e0, e1, e2, e3);
  reinterpret_cast<int4*>(bcur)[lane] = make_int4(e0, e1, e2, e3);
  if (lane == 31) bstart[kBuckets] = incl;
}

// bilinear combination of the sample's in-plane corners from a dense row (row points at the corner
// (h0, w0); corners outside the volume count as 0)
__device__ __forceinline__ float plane_bil(const float* row, int kst, const Rec& c, int H, int W) {
  const bool xok = c.w0 + 1 < W, yok = c.h0 + 1 < H;
  const float v00 = row[0];
  const float v01 = xok ? row[1] : 0.f;
  const float v10 = yok ? row[kst] : 0.f;
  const float v11 = (xok && yok) ? row[kst + 1] : 0.f;
  const float ax0 = 1.f - c.fw, ax1 = c.fw;
  return (1.f - c.fh) * fmaf(ax1, v01, ax0 * v00) + c.fh * fmaf(ax1, v11, ax0 * v10);
}

// adds round(value * w_c) (value already scaled) for the sample's in-volume corners to an int32 row
__device__ __forceinline__ void scatter_fixed_row(int* row, int k00, int ncw, const Rec& c, float sv, int H, int W) {
  const float ax0 = 1.f - c.fw, ax1 = c.fw, ay0 = 1.f - c.fh, ay1 = c.fh;
  const bool xok = c.w0 + 1 < W, yok = c.h0 + 1 < H;
  atomicAdd(row + k00, fix_round(sv * (ax0 * ay0)));
  if (xok) atomicAdd(row + k00 + 1, fix_round(sv * (ax1 * ay0)));
  if (yok) {
    atomicAdd(row + k00 + ncw, fix_round(sv * (ax0 * ay1)));
    if (xok) atomicAdd(row + k00 + ncw + 1, fix_round(sv * (ax1 * ay1)));
  }
}

// 16-key tiles of a chunk holding the sample's corners (rows h0, h0 + 1 of the chunk)
__device__ __forceinline__ uint32_t corner_tiles(int k00, int ncw, bool xok, bool yok) {
  uint32_t m = (1u << (k00 >> 4)) | (xok ? 1u << ((k00 + 1) >> 4) : 0u);
  if (yok) m |= (1u << ((k00 + ncw) >> 4)) | (xok ? 1u << ((k00 + ncw + 1) >> 4) : 0u);
  return m;
}

// The envelope walk: chunk (zr, iy, ix) covers frames zlo + zr * pg .. + pg - 1 (those up to zhi),
// rows [ya, yb] and columns [xa, xb] (windows of R rows / cw columns with one row / column of overlap,
// so that the four corners a sample has in a plane fall in one chunk).  Its keys are numbered
// pl * kpp + (y - ya) * kst + (x - xa) for chunk plane pl; m marks the 16-key tiles any sample of the
// tile touches (every tile of the chunk when no masks are kept; pg == 2 only with masks).  Tile masks
// are kept per plane for up to kMaskChunks chunks.
constexpr int kMaskChunks = 4;

struct Chunk {
  int zr, iy, ix;
  uint32_t m;
};

__device__ __forceinline__ int chunk_ya(const Env& E, const Chunk& k) { return E.ylo + k.iy * (E.R - 1); }
__device__ __forceinline__ int chunk_yb(const Env& E, const Chunk& k) { return min(chunk_ya(E, k) + E.R - 1, E.yhi); }
__device__ __forceinline__ int chunk_xa(const Env& E, const Chunk& k) { return E.xlo + k.ix * (E.cw - 1); }
__device__ __forceinline__ int chunk_xb(const Env& E, const Chunk& k) { return min(chunk_xa(E, k) + E.cw - 1, E.xhi); }

// the chunk's tile mask; 0 = nothing to do
__device__ __forceinline__ uint32_t chunk_mask(const Env& E, const uint32_t* mask, bool masks, const Chunk& k) {
  if (masks) {
    const int c = k.iy * E.nx + k.ix, z0 = k.zr * E.pg;
    uint32_t m = mask[(z0 + 1) * kMaskChunks + c];
    if (E.pg == 2 && E.zlo + z0 + 1 <= E.zhi) m |= mask[(z0 + 2) * kMaskChunks + c] << (E.kpp >> 4);
    return m;
  }
  const int ntile = ((chunk_yb(E, k) - chunk_ya(E, k) + 1) * E.kst + 15) >> 4;
  return ntile >= 32 ? 0xffffffffu : (1u << ntile) - 1u;
}

// moves k to the first chunk at or after it with a touched tile; false when the walk is over
// (nz = frames of the envelope, 0 when the tile has no work)
__device__ __forceinline__ bool chunk_seek(const Env& E, const uint32_t* mask, bool masks, int nz, Chunk& k) {
  const int ng = E.pg == 2 ? (nz + 1) >> 1 : nz;  // chunk rows along z
  while (k.zr < ng) {
    k.m = chunk_mask(E, mask, masks, k);
    if (k.m) return true;
    if (++k.ix == E.nx) {
      k.ix = 0;
      if (++k.iy == E.ny) {
        k.iy = 0;
        ++k.zr;
      }
    }
  }
  return false;
}
__device__ __forceinline__ bool chunk_first(const Env& E, const uint32_t* mask, bool masks, int nz, Chunk& k) {
  k.zr = k.iy = k.ix = 0;
  return chunk_seek(E, mask, masks, nz, k);
}
__device__ __forceinline__ bool chunk_next(const Env& E, const uint32_t* mask, bool masks, int nz, Chunk& k) {
  if (++k.ix == E.nx) {
    k.ix = 0;
    if (++k.iy == E.ny) {
      k.iy = 0;
      ++k.zr;
    }
  }
  return chunk_seek(E, mask, masks, nz, k);
}

// Row of chunk key `key` in the K/V buffers of the sample, -1 past the chunk and outside the volume /
// K-V window.
__device__ __forceinline__ int chunk_key_row(const AttnParams& P, const Env& E, const Chunk& k, int key) {
  const int pl = (E.pg == 2 && key >= E.kpp) ? 1 : 0;
  key -= pl * E.kpp;
  // key / kst exactly: (key + 0.5) / kst is at least 1 / (2 kst) away from an integer
  const int ky = static_cast<int>((static_cast<float>(key) + 0.5f) * (1.f / static_cast<float>(E.kst)));
  const int y = chunk_ya(E, k) + ky, x = chunk_xa(E, k) + (key - ky * E.kst);
  const int z = E.zlo + k.zr * E.pg + pl, zl = z - P.kv_frame0;
  const bool ok = y <= chunk_yb(E, k) && x <= chunk_xb(E, k) && z <= E.zhi && zl >= 0 && zl < P.kv_frames && y >= 0 &&
                  y < P.H && x >= 0 && x < P.W;
  return ok ? (zl * P.H + y) * P.W + x : -1;
}

// cp.async path: starts the copy of the chunk's keys in the tiles of k.m into kbuf rows (lanes along
// the 16-byte pieces of a row); rows without a key are zeroed.  The copies land at the caller's
// cp_async_wait_all().
template <int DCH>
__device__ __forceinline__ void issue_keys(const AttnParams& P, const TileCtx& T, const Env& E, const Chunk& k,
                                           __nv_bfloat16* kbuf, int rs, const __nv_bfloat16* base, long long ld) {
  const __nv_bfloat16* gb = base + static_cast<long long>(T.b) * P.Nkv * ld + T.head * P.d;
  const int items = __popc(k.m) * 16 * DCH;
  for (int idx = threadIdx.x; idx < items; idx += kThreads) {
    const int slot = idx / DCH, ch = idx - slot * DCH;  // DCH is a constant: multiply-shift
    const int key = nth_bit(k.m, slot >> 4) * 16 + (slot & 15);
    __nv_bfloat16* dst = kbuf + static_cast<size_t>(key) * rs + ch * 8;
    const int row = chunk_key_row(P, E, k, key);
    if (row >= 0)
      cp_async16(smem_u32(dst), gb + static_cast<long long>(row) * ld + ch * 8);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Tensor maps of one launch: K and V, box widths 8, 16, 24 and 32 keys (index j = kst / 8 - 1) and
// heights 1, 2, 4 and 8 key rows (index h); bit 4 j + h of `have` set when map [j][h] of both exists.
struct alignas(64) KeyMaps {
  CUtensorMap k[4][4], v[4][4];
  int have;
};

// Fills the launch's tensor maps (widths whose box fits the volume; 16-byte aligned K / V base and row
// stride).  False when TMA cannot serve the launch (the kernels then load with cp.async).
bool make_key_maps(KeyMaps* maps, const AttnParams& P, int rs);

// TMA path: the last four warps copy, for each chunk plane pl, rows [ya, yb] x columns [xa, xa + kst) into kbuf
// rows pl * kpp + (y - ya) * kst + x - xa.  With the maps of the chunk width a plane's nr rows take
// nr / 8 boxes of 8 rows and one box per set bit of nr % 8 (4, 2, 1 rows; heights never exceed nr <= H,
// so their maps exist); without a map of that width, one 8-key box per row segment.  Boxes whose keys
// are all in untouched tiles are skipped; coordinates outside the volume / K-V window read as zeros,
// and the half tile past a plane's last key, when the plane ends inside a touched tile, is filled by
// one more 8-key box placed wholly outside the volume (zeros).  The copies complete on mbarrier `bar`.
// In TMA mode the key buffer is written only by TMA, and its earlier generic reads are ordered by the
// CTA barrier before the call; `first` adds the proxy fence for the setup's generic use of the buffer.
// (boxes <= maxkeys / 8 <= 64: two per lane)
__device__ __forceinline__ void issue_keys_tma(const AttnParams& P, const TileCtx& T, const Env& E, const Chunk& k,
                                               __nv_bfloat16* kbuf, int rs, const CUtensorMap (*maps)[4], int have,
                                               uint32_t bar, bool first) {
  // box b is issued by warp kW0 + b % 4: a warp's copies issue one lane after another, so four warps
  // shorten the issue (measured: 4 ~ 8 warps > 16 > 1); the last four warps, which have the least
  // work in the phases the copies overlap (hit loops, zeroing, conversions stride from thread 0)
  constexpr int kIW = 4, kW0 = kWarps - kIW;
  if (threadIdx.x < 32 * kW0) return;
  const int lane = threadIdx.x & 31, wid = (threadIdx.x >> 5) - kW0;
  // bit 31 of `have` (set only by the MSL_TEST_TMA_NO_COPY=1 test hook): arm the barrier's byte count
  // but issue no copy, so the bounded wait runs out with nothing in flight
  const bool nocopy = have < 0;
  const int nr = chunk_yb(E, k) - chunk_ya(E, k) + 1;  // rows of one plane
  const int nkeys = nr * E.kst;                         // keys of one plane
  const int mi = (E.kst >> 3) - 1;
  const int hm = mi < 4 ? (have >> (4 * mi)) & 15 : 0;  // heights available at this width
  const int need = (nr >= 8 ? 8 : 0) | (nr & 7);        // heights the row decomposition uses
  const bool wide = hm & 1;
  const bool multi = wide && (need & ~hm) == 0;
  const int nbp = multi ? (nr >> 3) + __popc(nr & 7) : (wide ? nr : nkeys >> 3);  // boxes per plane
  const int np = E.pg == 2 && E.zlo + k.zr * 2 + 1 <= E.zhi ? 2 : 1;
  // boxes b = lane and lane + 32 (plane b / nbp): first row, rows, first column, keys per row, map
  bool on[2];
  int brow[2], bh[2], bcol[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int b = lane + 32 * u;
    on[u] = false;
    brow[u] = 0, bh[u] = 1, bcol[u] = 0;
    if (b < np * nbp) {
      const int pl = b >= nbp ? 1 : 0, lb = b - pl * nbp;
      if (multi) {
        if (lb < (nr >> 3)) {
          brow[u] = 8 * lb;
          bh[u] = 8;
        } else {
          int r0 = nr & ~7, kk = lb - (nr >> 3);
          for (int bit = 4; bit >= 1; bit >>= 1) {
            if (!(nr & bit)) continue;
            if (kk == 0) {
              bh[u] = bit;
              break;
            }
            r0 += bit;
            --kk;
          }
          brow[u] = r0;
        }
      } else if (wide) {
        brow[u] = lb;
      } else {
        brow[u] = lb / (E.kst >> 3);
        bcol[u] = (lb - brow[u] * (E.kst >> 3)) * 8;
      }
      const int key0 = pl * E.kpp + brow[u] * E.kst + bcol[u];
      const int key1 = key0 + (wide ? bh[u] * E.kst : 8) - 1;
      const int t0 = key0 >> 4, t1 = key1 >> 4;
      on[u] = ((k.m >> t0) & ((2u << (t1 - t0)) - 1u)) != 0u;
    }
  }
  // plane pl's tail: keys pl * kpp + nkeys .. +7 when that tile is touched
  bool tail[2];
#pragma unroll
  for (int pl = 0; pl < 2; ++pl) {
    const int kt = pl * E.kpp + nkeys;
    tail[pl] = pl < np && (nkeys & 15) && ((k.m >> (kt >> 4)) & 1u);
  }
  const int bw = wide ? E.kst : 8;  // keys per box row
  const int rows_on = __reduce_add_sync(0xffffffffu, (on[0] ? bh[0] : 0) + (on[1] ? bh[1] : 0));
  if (threadIdx.x == 32 * kW0) {
    if (first) fence_proxy_async();
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>((rows_on * bw + ((tail[0] ? 8 : 0) + (tail[1] ? 8 : 0))) * rs * 2));
  }
  __syncwarp();
  if (first && (on[0] || on[1])) fence_proxy_async();
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    if (nocopy || !on[u] || (lane + 32 * u) % kIW != wid) continue;
    const int b = lane + 32 * u;
    const int pl = b >= nbp ? 1 : 0;
    const int hi = bh[u] == 8 ? 3 : (bh[u] == 4 ? 2 : (bh[u] == 2 ? 1 : 0));
    tma_load_5d(smem_u32(kbuf) + static_cast<uint32_t>((pl * E.kpp + brow[u] * E.kst + bcol[u]) * rs * 2),
                wide ? &maps[mi][hi] : &maps[0][0], bar, T.head * P.d, chunk_xa(E, k) + bcol[u],
                chunk_ya(E, k) + brow[u], E.zlo + k.zr * E.pg + pl - P.kv_frame0, T.b);
  }
  if (!nocopy && wid == 0 && lane < 2 && tail[lane])  // columns W .. W+7: all outside the volume
    tma_load_5d(smem_u32(kbuf) + static_cast<uint32_t>((lane * E.kpp + nkeys) * rs * 2), &maps[0][0], bar,
                T.head * P.d, P.W, 0, 0, T.b);
}

// Waits for the TMA copies of phase `parity` on mbarrier bar.  Bounded: after about a second the CTA
// stops waiting and issuing (flag *dead, status MSL_STATUS_TIMEOUT); the thread that gave up then
// waits once more, again for at most about a second, for the copies of that phase that were issued
// (no later phase issues any), so that none lands in shared memory the SM may already have given to
// the next CTA.  After the CTA barrier that follows every wait, the chunk loops read *dead
// (tile_dead) and leave before any phase that reads the key buffer; the tile's results are invalid.
__device__ __forceinline__ void wait_keys(uint32_t bar, uint32_t parity, volatile int* dead, uint32_t* status) {
  if (mbar_try_wait(bar, parity) || *dead) return;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*dead) return;
    if (global_ns() - t0 > 1000000000ull) {
      *dead = 1;
      if (status) atomicOr(status, MSL_STATUS_TIMEOUT);
      const unsigned long long t1 = global_ns();
      while (!mbar_try_wait(bar, parity) && global_ns() - t1 < 1000000000ull) {
      }
      return;
    }
  }
}

// true once a TMA wait of this CTA gave up (read after a CTA barrier: the same on every thread)
__device__ __forceinline__ bool tile_dead(const int* dead) { return *reinterpret_cast<const volatile int*>(dead) != 0; }

// zeroes rows 0..ROWS-1 of the 16-key tiles of mask m in a dense fp32 / int32 tile
template <int ROWS>
__device__ __forceinline__ void zero_tiles(float* buf, int sld, uint32_t m) {
  // one warp per 16-key tile (one bit search per warp and tile); a store instruction covers 8 rows x
  // 64 bytes: 4 wavefronts, the minimum for 512 bytes
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = __popc(m);
  for (int o = warp; o < nt; o += kWarps) {
    float* const col = buf + nth_bit(m, o) * 16 + (lane & 3) * 4;
#pragma unroll
    for (int row = lane >> 2; row < ROWS; row += 8)
      *reinterpret_cast<float4*>(col + static_cast<size_t>(row) * sld) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// S / dP for the 16 queries of a row group over the chunk's tiles of mask m: A = 16 staged bf16
// rows xs (Q or dO, row stride rs) read with ldmatrix, kbuf rows (keys) with ldmatrix; the WPG warps
// of the group split the tiles round robin (`part` = warp index within the group).
template <int DCH, int WPG>
__device__ __forceinline__ void dense_tiles(const __nv_bfloat16* kbuf, const __nv_bfloat16* xs, int rs, float* srow,
                                            int sld, int part, uint32_t m) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  const int nt = __popc(m);
  if (part >= nt) return;
  uint32_t qa[DCH / 2 > 0 ? DCH / 2 : 1][4], qt[2] = {0u, 0u};
  {
    const __nv_bfloat16* ap = xs + static_cast<size_t>(lane & 15) * rs + (lane >> 4) * 8;
#pragma unroll
    for (int ks = 0; ks < DCH / 2; ++ks) ldsm_x4(smem_u32(ap + ks * 16), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
    if constexpr (DCH & 1) ldsm_x2(smem_u32(xs + static_cast<size_t>(lane & 15) * rs + (DCH - 1) * 8), qt[0], qt[1]);
  }
  for (int o = part; o < nt; o += WPG) {
    const int gi = nth_bit(m, o);
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    const int key = gi * 16 + rr + ((mi >> 1) ? 8 : 0);
    const __nv_bfloat16* rowp = kbuf + static_cast<size_t>(key) * rs + ((mi & 1) ? 8 : 0);
#pragma unroll
    for (int ks = 0; ks < DCH / 2; ++ks) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(rowp + ks * 16), b0, b1, b2, b3);
      mma16816(c0, qa[ks], b0, b1);
      mma16816(c1, qa[ks], b2, b3);
    }
    if constexpr (DCH & 1) {
      const int key2 = gi * 16 + rr + ((mi & 1) ? 8 : 0);
      uint32_t e0, e1;
      ldsm_x2(smem_u32(kbuf + static_cast<size_t>(key2) * rs + (DCH - 1) * 8), e0, e1);
      mma1688(c0, qt[0], qt[1], e0);
      mma1688(c1, qt[0], qt[1], e1);
    }
    float* p0 = srow + static_cast<size_t>(g) * sld + gi * 16 + 2 * t4;
    float* p1 = srow + static_cast<size_t>(g + 8) * sld + gi * 16 + 2 * t4;
    *reinterpret_cast<float2*>(p0) = make_float2(c0[0], c0[1]);
    *reinterpret_cast<float2*>(p1) = make_float2(c0[2], c0[3]);
    *reinterpret_cast<float2*>(p0 + 8) = make_float2(c1[0], c1[1]);
    *reinterpret_cast<float2*>(p1 + 8) = make_float2(c1[2], c1[3]);
  }
}

// loads G extra keys / values of this head into kbuf rows 0..G-1 (zero up to gp)
template <int DCH>
__device__ __forceinline__ void load_extra(const AttnParams& P, const TileCtx& T, __nv_bfloat16* kbuf, int rs,
                                           const void* src, int gp) {
  const __nv_bfloat16* eb = static_cast<const __nv_bfloat16*>(src) + static_cast<long long>(T.b) * P.G * P.e_ld +
                            T.head * P.d;
  for (int idx = threadIdx.x; idx < gp * DCH; idx += kThreads) {
    const int key = idx / DCH, ch = idx - (idx / DCH) * DCH;
    __nv_bfloat16* dst = kbuf + static_cast<size_t>(key) * rs + ch * 8;
    if (key < P.G)
      cp_async16(smem_u32(dst), eb + static_cast<long long>(key) * P.e_ld + ch * 8);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
  }
  cp_async_wait_all();
}

// ------------------------------------------------------------------------------ 32-query tiles
// Geometry shared by the kernels that use 4 x 8 query tiles (two 16-query row groups, 8 warps each,
// 16 lanes per query for the per-sample work).
namespace t32 {
constexpr int kGroups = 2;                  // 16-query row groups per tile
constexpr int kWPG = kWarps / kGroups;      // warps per row group
constexpr int kLPQ = kWPG * 32 / 16;        // lanes per query
constexpr int kTileH = 4, kQ = kTileH * kTileW;
constexpr int kTRow = 40;                   // bf16 per key row of a transposed dense tile (32 + 8 pad)
constexpr int kMaxKeys = 256;               // backward chunk cap: 16 tiles of 16 keys
constexpr int kMaxKeysFwd = 512;            // forward chunk cap: 32 tiles (the whole tile mask)
constexpr int kMaxMaskChunks = kMaskChunks;  // chunks per plane with their own tile masks
constexpr float kFixRange = 2097152.f;      // 2^21: fixed-point full scale of a dense row



// In-place conversion of the tiles of mask m of an int32 dense tile [32][sld] (fixed point, per-row
// inverse scale inv[q]) into bf16 [key][kTRow].  Two phases separated by a barrier; every thread of
// the CTA must call it.  Item = (key, half): 16 queries of one key; MAXKEYS = the launch's key cap.
template <int MAXKEYS>
__device__ __forceinline__ void transpose_fixed(float* buf, int sld, uint32_t m, const float* inv) {
  constexpr int kMaxIt = MAXKEYS * 2 / kThreads;
  const int* src = reinterpret_cast<const int*>(buf);
  const int items = __popc(m) * 32;
  uint32_t hold[kMaxIt][8];
  int keyv[kMaxIt];  // the item's key, found once (bit search) for both phases
#pragma unroll
  for (int u = 0; u < kMaxIt; ++u) {
    const int i = threadIdx.x + u * kThreads;
    keyv[u] = 0;
    if (i < items) {
      const int key = nth_bit(m, i >> 5) * 16 + (i & 15), half = (i >> 4) & 1;
      keyv[u] = key;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int q = half * 16 + 2 * e;
        const float f0 = fix_float(src[static_cast<size_t>(q) * sld + key]) * inv[q];
        const float f1 = fix_float(src[static_cast<size_t>(q + 1) * sld + key]) * inv[q + 1];
        hold[u][e] = pack_bf16(f0, f1);
      }
    }
  }
  __syncthreads();
  uint32_t* dst = reinterpret_cast<uint32_t*>(buf);
#pragma unroll
  for (int u = 0; u < kMaxIt; ++u) {
    const int i = threadIdx.x + u * kThreads;
    if (i < items) {
      const int key = keyv[u], half = (i >> 4) & 1;
      uint4* d = reinterpret_cast<uint4*>(dst + key * (kTRow / 2) + half * 8);
      d[0] = make_uint4(hold[u][0], hold[u][1], hold[u][2], hold[u][3]);
      d[1] = make_uint4(hold[u][4], hold[u][5], hold[u][6], hold[u][7]);
    }
  }
}

// o[16 queries of group r][channel tiles nt0..nt1) += A . kbuf over the tiles of mask m; A = rows of
// the transposed bf16 tile tb ([key][query]) read with ldmatrix.trans, kbuf rows through
// ldmatrix.trans.
// With KSPLIT > 1 the warp takes every KSPLIT-th touched tile from the kpar-th on (the partial sums
// of the KSPLIT warps that share channels are added by the caller).
template <int DCH, int TPW, int KSPLIT = 1>
__device__ __forceinline__ void dq_product(const __nv_bfloat16* tb, int r, const __nv_bfloat16* kbuf, int rs, int nt0,
                                           int nt1, uint32_t m, float (&o)[TPW + 1][4], int kpar = 0) {
  const int lane = threadIdx.x & 31;
  const int mi = lane >> 3, rr = lane & 7;
  if (KSPLIT > 1) {  // drop the touched tiles of the other warps: keep ordinals kpar, kpar + KSPLIT, ...
    uint32_t keep = 0u;
    int ord = 0;
    for (uint32_t mm = m; mm; mm &= mm - 1u, ++ord)
      if (ord % KSPLIT == kpar) keep |= mm & (~mm + 1u);
    m = keep;
  }
  for (uint32_t mm = m; mm; mm &= mm - 1u) {
    const int kk = __ffs(mm) - 1;
    uint32_t a[4];
    // matrices: (queries 0-7, keys 0-7) (q 8-15, k 0-7) (q 0-7, k 8-15) (q 8-15, k 8-15) of the group
    const __nv_bfloat16* ap = tb + static_cast<size_t>(kk * 16 + rr + ((mi >> 1) ? 8 : 0)) * kTRow + r * 16 +
                              ((mi & 1) ? 8 : 0);
    ldsm_x4_t(smem_u32(ap), a[0], a[1], a[2], a[3]);
    const __nv_bfloat16* rowp = kbuf + static_cast<size_t>(kk * 16 + rr + ((mi & 1) ? 8 : 0)) * rs;
#pragma unroll
    for (int jj = 0; jj < TPW; jj += 2) {
      const int nt = nt0 + jj;
      if (nt + 1 < nt1) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(rowp + (nt + (mi >> 1)) * 8), b0, b1, b2, b3);
        mma16816(o[jj], a, b0, b1);
        mma16816(o[jj + 1], a, b2, b3);
      } else if (nt < nt1) {
        uint32_t b0, b1;
        ldsm_x2_t(smem_u32(rowp + nt * 8), b0, b1);
        mma16816(o[jj], a, b0, b1);
      }
    }
  }
}

// The tile's queries through the CUDA-core gather (dsa_simt.cuh), forward (BWD false: out, lse) or
// backward (dq, d(offsets), dK / dV atomics into the float32 accumulators): used when the tile's key
// envelope does not fit the sample records (temporal span over 29 frames, or over 255 rows or columns).
// The forward and the backward take this decision from the same envelope, so a tile runs the same
// formulation both ways.  Every thread of the CTA calls it; warp w takes queries w and w + 16.
// (The backward runs it in its own kernel, dsa_bwd_tc_fallback_kernel: inlined into the tensor-core
// backward, its register demand changed that kernel's register allocation, +2% measured, and called out
// of line it forced the kernel's parameters into local memory, +50%.)  NWARPS = warps of the caller.
template <int DCH, bool BWD, int NWARPS = kWarps>
__device__ __forceinline__ void tile_fallback(const AttnParams& P, const TileCtx& T) {
  constexpr int MAXC = (DCH + 3) / 4;
  const int warp = threadIdx.x >> 5;
  for (int q = warp; q < kQ; q += NWARPS) {
    int qh, qw;
    query_hw(T, q >> 4, q & 15, qh, qw);
    if (qh >= P.H || qw >= P.W) continue;  // warp-uniform
    QueryPos qp;
    qp.b = T.b;
    qp.head = T.head;
    qp.tg = T.tg;
    qp.h = qh;
    qp.w = qw;
    qp.r = (static_cast<long long>(T.tl) * P.H + qh) * P.W + qw;
    if constexpr (BWD)
      bwd_query<__nv_bfloat16, 8, MAXC>(P, qp);
    else
      fwd_query<__nv_bfloat16, 8, MAXC>(P, qp);
  }
}

// true when the tile's envelope [zlo, zhi] x [ylo, yhi] x [xlo, xhi] exceeds what the sample records
// encode (t0 - zlo + 1 in 5 bits, h0 - ylo and w0 - xlo in 8 bits): the CUDA-core fallback takes it
__device__ __forceinline__ bool env_overflow(int zlo, int zhi, int ylo, int yhi, int xlo, int xhi) {
  const bool any = zlo <= zhi && ylo <= yhi && xlo <= xhi;
  return any && (zhi - zlo + 2 > 31 || yhi - ylo > 255 || xhi - xlo > 255);
}

}  // namespace t32

}  // namespace tc
}  // namespace msl
