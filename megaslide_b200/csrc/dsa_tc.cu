// Tensor-core ("key envelope") formulation of the deformable gather attention forward, bf16.
//
// One CTA owns a tile of 4 x 8 queries of one frame, one head and one sample (32 queries = two
// 16-query row groups; 16 warps, 8 per group; 16 lanes per query for the per-query work).
// Every trilinear corner any of the tile's samples can touch lies in the tile's key envelope:
// frames [zlo, zhi] x rows [ylo, yhi] x columns [xlo, xhi].  The CTA walks it one frame ("plane")
// at a time, in chunks of at most `maxkeys` keys (rows and columns split with one row / column of
// overlap so that the four corners a sample has in a plane always fall in one chunk):
//
//   pass 1, per chunk:  S = Q . K_chunk^T on the tensor cores (mma.sync bf16 -> fp32) over the
//                       16-key tiles any corner touches; every sample with corners in the chunk adds
//                       sum_corners w_c * S[q, corner] to its score.
//   softmax:            per query over its K samples (+ G extra keys, scored the same way).
//   pass 2, per chunk:  every sample scatters p * w_c into a dense P~[q, key] (32-bit fixed point,
//                       per-query scale), converted once to bf16 [key][query]; O += P~ . V_chunk on
//                       the tensor cores (ldmatrix.trans for both operands).
//
// The setup sorts the tile's active samples into one list by frame (counting sort), so the samples
// with a corner in a plane are one contiguous range that all 512 threads stride through, and records
// per (plane, chunk) which 16-key tiles any corner touches: loads, products and the conversion visit
// only those.  Sample coordinates come from the offsets with the same float32 arithmetic as the
// CUDA-core kernels (msl_common.cuh), so corner choices are identical; each sample's corner and
// trilinear fractions are kept as a packed 8-byte record (fractions quantised to 12 bits:
// interpolation weights within 1.2e-4 - this path is bf16 only).
// Reference semantics: infinity/video/attention.py:113-186 (grid, grid_sample, softmax, dropout,
// value sum) and :159-173 (extra keys).

#include "dsa_tc.cuh"

#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

namespace msl {
namespace tc {
namespace fwd {

using namespace t32;

struct Smem {
  __nv_bfloat16* kbuf;      // [maxkeys][rs]   K or V chunk (setup: staged offsets, spilling into sbuf)
  float* sbuf;              // [32][sld]       S (fp32), then P~ (int32), then P~^T (bf16 [key][40])
  __nv_bfloat16* qs;        // [32][rs]        Q rows of the tile
  unsigned long long* rec;  // [32][K]         packed sample records
  float* sacc;              // [32][K + G]     scores, then unnormalised dropout-applied weights
  int* env;                 // envelope + base-grid tables
  float* lrow;              // [32]            softmax sums
  float* qsc;               // [2][32]         P~ fixed-point scale / inverse per query
  int* bstart;              // [132]           hit list: first entry of each (chunk, frame) bucket (+ end)
  int* bcur;                // [128]           bucket counts, then fill cursors
  uint32_t* mask;           // [32][4]         16-key tiles touched per (plane, chunk)
  unsigned short* hits;     // [32 * K]        sample indices q * K + j sorted by frame bucket
  unsigned long long* kbar; // mbarrier of the key buffer's TMA copies
  int* dead;                // set when a TMA wait gave up
};

__device__ __forceinline__ Smem carve(unsigned char* base, const AttnParams& P, const TcLaunch& L) {
  Smem s;
  size_t off = 0;
  s.kbuf = reinterpret_cast<__nv_bfloat16*>(base + off);
  off += static_cast<size_t>(L.maxkeys) * L.rs * 2;
  s.sbuf = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * L.sld * 4;
  s.qs = reinterpret_cast<__nv_bfloat16*>(base + off);
  off += static_cast<size_t>(kQ) * L.rs * 2;
  s.rec = reinterpret_cast<unsigned long long*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 8;
  s.sacc = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * (P.K + P.G) * 4;
  s.env = reinterpret_cast<int*>(base + off);
  off += kEnvWords * 4;
  s.lrow = reinterpret_cast<float*>(base + off);
  off += kQ * 4;
  s.qsc = reinterpret_cast<float*>(base + off);
  off += 2 * kQ * 4;
  s.bstart = reinterpret_cast<int*>(base + off);
  off += (kBuckets + 4) * 4;
  s.bcur = reinterpret_cast<int*>(base + off);
  off += kBuckets * 4;
  s.mask = reinterpret_cast<uint32_t*>(base + off);
  off += 32 * kMaxMaskChunks * 4;
  s.hits = reinterpret_cast<unsigned short*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 2;
  // last: the setup's offset staging spills from the key buffer into the regions after it
  off = (off + 7) & ~static_cast<size_t>(7);
  s.kbar = reinterpret_cast<unsigned long long*>(base + off);
  s.dead = reinterpret_cast<int*>(base + off + 8);
  return s;
}

// shared memory besides the key buffer and the dense tile
size_t smem_fixed(const AttnParams& P, int rs) {
  return static_cast<size_t>(kQ) * rs * 2 + static_cast<size_t>(kQ) * P.K * (8 + 2) +
         static_cast<size_t>(kQ) * (P.K + P.G) * 4 + kEnvWords * 4 + kQ * 4 * 3 + (2 * kBuckets + 4 + 32 * kMaxMaskChunks) * 4 +
         24 + 256;
}

// P~ . V: channel groups of a row group's 8 warps (all channel tiles per warp up to head_dim 72; two
// groups above, for registers)
__host__ __device__ constexpr int pv_channel_groups(int dch) { return dch <= 9 ? 1 : 2; }

template <int DCH>
__global__ void __launch_bounds__(kThreads, 1) dsa_fwd_tc_kernel(const AttnParams P, const TcLaunch L,
                                                                  const __grid_constant__ KeyMaps maps) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const Smem S = carve(smem_raw, P, L);
  const TileCtx T = decode_tile(P, L, kTileH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp / kWPG, part = warp - (warp / kWPG) * kWPG;
  const int ll = part * 32 + lane;
  const int cq = ll / kLPQ, sub = ll - (ll / kLPQ) * kLPQ;
  const int K = P.K, KG = P.K + P.G;
  // setup: the lanes of a query own contiguous window ranges [js, je)
  const int jper = (K + kLPQ - 1) / kLPQ;
  const int js = min(K, sub * jper), je = min(K, js + jper);
  const int n = je - js;
  const int qi = r * 16 + cq;
  const float invK = 1.f / static_cast<float>(K);

  int qh, qw;
  query_hw(T, r, cq, qh, qw);
  const bool qvalid = qh < P.H && qw < P.W;
  const long long qrow = (static_cast<long long>(T.tl) * P.H + qh) * P.W + qw;
  const int qbase = qi * K;  // this query's records
  float* sacc = S.sacc + static_cast<size_t>(qi) * KG;

  float* tabz = reinterpret_cast<float*>(S.env + 16);
  float* taby = tabz + 96;
  float* tabx = taby + 96;
  if (threadIdx.x == 0) {
    S.env[0] = 0x7fffffff; S.env[1] = -0x7fffffff; S.env[2] = 0x7fffffff;
    S.env[3] = -0x7fffffff; S.env[4] = 0x7fffffff; S.env[5] = -0x7fffffff;
  }
  if (threadIdx.x < kBuckets) S.bcur[threadIdx.x] = 0;
  if (threadIdx.x < 32 * kMaxMaskChunks) S.mask[threadIdx.x] = 0u;
  // TMA destinations are 128-byte aligned: boxes start at multiples of 8 keys x rs (rs % 8 == 0) bf16
  const bool tma = L.tma && (smem_u32(S.kbuf) & 127u) == 0u;
  const uint32_t kbar = smem_u32(S.kbar);
  if (threadIdx.x == 0) {
    *S.dead = 0;
    if (tma) {
      mbar_init(kbar, 1);
      fence_mbar_init();
    }
  }
  uint32_t kphase = 0;
  fill_tabs(P, T, kTileH, tabz, taby, tabx);

  // ---- stage the tile's offsets (this head) and Q rows with one wave of cp.async.  An offsets row
  //      (3K floats at any 4-byte alignment) lands at row base + its misalignment so that its 16-byte
  //      aligned body copies with 16-byte cp.async; the up to 3 floats before and after it with 4-byte
  //      ones (no byte outside the row is read).
  const int K3 = 3 * K;
  const int OS = (K3 + 3 + 3) & ~3;  // staged row stride (floats): 16-byte aligned rows
  float* ostage = reinterpret_cast<float*>(S.kbuf);
  float* bstage = ostage + static_cast<size_t>(kQ) * OS;  // this head's offset bias (K3 floats), if any
  if (P.off_bias)
    for (int e = threadIdx.x; e < K3; e += kThreads)
      cp_async4(smem_u32(bstage + e), P.off_bias + static_cast<long long>(T.head) * K3 + e);
  // misalignment (floats) of this thread's own query row, where its staged row starts
  const int omis = static_cast<int>(
      (reinterpret_cast<uintptr_t>(P.offsets + (static_cast<long long>(T.b) * P.Nq + qrow) * P.off_ld +
                                   static_cast<long long>(T.head) * K3) >> 2) & 3u);
  for (int q2 = warp; q2 < kQ; q2 += kWarps) {
    int sqh, sqw;
    query_hw(T, q2 >> 4, q2 & 15, sqh, sqw);
    const bool ok = sqh < P.H && sqw < P.W;
    const long long grow = static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + sqh) * P.W + sqw;
    if (ok) {
      const float* src = P.offsets + grow * P.off_ld + static_cast<long long>(T.head) * K3;
      const int mis = static_cast<int>((reinterpret_cast<uintptr_t>(src) >> 2) & 3u);
      const int lead = (4 - mis) & 3, nb = (K3 - lead) >> 2, tail0 = lead + 4 * nb;
      float* dst = ostage + static_cast<size_t>(q2) * OS + mis;  // dst + lead is 16-byte aligned
      if (lane < lead) cp_async4(smem_u32(dst + lane), src + lane);
      for (int c = lane; c < nb; c += 32) cp_async16(smem_u32(dst + lead + 4 * c), src + lead + 4 * c);
      if (tail0 + lane < K3) cp_async4(smem_u32(dst + tail0 + lane), src + tail0 + lane);
    }
    for (int ch = lane; ch < DCH; ch += 32) {
      __nv_bfloat16* dq_ = S.qs + static_cast<size_t>(q2) * L.rs + ch * 8;
      if (ok)
        cp_async16(smem_u32(dq_), static_cast<const __nv_bfloat16*>(P.q) + grow * P.q_ld + T.head * P.d + ch * 8);
      else
        *reinterpret_cast<uint4*>(dq_) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  const Tabs tb{tabz, taby, tabx};
  const int qy = qh - T.qh0, qx = qw - T.qw0;

  // ---- sample coordinates -> envelope (raw coordinates parked in rec / sacc)
  const int kvlo = max(P.kv_frame0, 0), kvhi = min(P.kv_frame0 + P.kv_frames, P.T) - 1;
  int zmn = 0x7fffffff, zmx = -0x7fffffff, ymn = 0x7fffffff, ymx = -0x7fffffff, xmn = 0x7fffffff, xmx = -0x7fffffff;
  bool miss = false;
  if (qvalid) {
    const float* oq = ostage + static_cast<size_t>(qi) * OS + omis;
    WinIdx wi;
    wi.init(js, P.kh, P.kw);
    for (int j = js; j < je; ++j, wi.advance(1, P.kh, P.kw)) {
      float pt, ph, pw;
      float o0 = oq[3 * j], o1 = oq[3 * j + 1], o2 = oq[3 * j + 2];
      if (P.off_bias) {  // the lanes of the query pair read the same bias words: broadcasts
        o0 = __fadd_rn(o0, bstage[3 * j]);
        o1 = __fadd_rn(o1, bstage[3 * j + 1]);
        o2 = __fadd_rn(o2, bstage[3 * j + 2]);
      }
      tab_coords(P, tb, qy, qx, wi.it, wi.ih, wi.iw, o0, o1, o2, pt, ph, pw);
      S.rec[qbase + j] = (static_cast<unsigned long long>(__float_as_uint(ph)) << 32) | __float_as_uint(pt);
      sacc[j] = pw;
      const int t0 = static_cast<int>(floorf(pt)), h0 = static_cast<int>(floorf(ph)), w0 = static_cast<int>(floorf(pw));
      for (int dt = 0; dt < 2; ++dt) {
        const int tc = t0 + dt;
        if (tc >= P.T) continue;
        if (tc < kvlo || tc > kvhi) {
          miss = true;
          continue;
        }
        zmn = min(zmn, tc);
        zmx = max(zmx, tc);
      }
      ymn = min(ymn, h0);
      ymx = max(ymx, h0 + 1 < P.H ? h0 + 1 : h0);
      xmn = min(xmn, w0);
      xmx = max(xmx, w0 + 1 < P.W ? w0 + 1 : w0);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    zmn = min(zmn, __shfl_xor_sync(kFull, zmn, o));
    zmx = max(zmx, __shfl_xor_sync(kFull, zmx, o));
    ymn = min(ymn, __shfl_xor_sync(kFull, ymn, o));
    ymx = max(ymx, __shfl_xor_sync(kFull, ymx, o));
    xmn = min(xmn, __shfl_xor_sync(kFull, xmn, o));
    xmx = max(xmx, __shfl_xor_sync(kFull, xmx, o));
  }
  if (lane == 0) {
    atomicMin(S.env + 0, zmn); atomicMax(S.env + 1, zmx);
    atomicMin(S.env + 2, ymn); atomicMax(S.env + 3, ymx);
    atomicMin(S.env + 4, xmn); atomicMax(S.env + 5, xmx);
  }
  if (__any_sync(kFull, miss) && lane == 0 && P.status) atomicOr(P.status, MSL_STATUS_HALO_MISS);
  __syncthreads();
  Env E;
  E.zlo = S.env[0]; E.zhi = S.env[1]; E.ylo = S.env[2]; E.yhi = S.env[3]; E.xlo = S.env[4]; E.xhi = S.env[5];
  const bool any = E.zlo <= E.zhi && E.ylo <= E.yhi && E.xlo <= E.xhi;
  if (any) {
    chunk_shape(E, L.maxkeys);
  } else {
    E.cw = E.R = E.ny = E.nx = 1;
    E.kst = 8;
  }
  const bool split = E.ny * E.nx > 1;
  // records hold t0 - zlo + 1 in 5 bits and h0 - ylo, w0 - xlo in 8 bits
  const bool overflow = env_overflow(E.zlo, E.zhi, E.ylo, E.yhi, E.xlo, E.xhi);
  if (overflow && threadIdx.x == 0 && P.status) atomicOr(P.status, MSL_STATUS_TC_RANGE);
  const bool work = any && !overflow;
  const bool masks = work && E.ny * E.nx <= kMaxMaskChunks;
  const bool fsplit = split && !masks;  // chunks of a plane share one hit bucket: filter the hits
  if (masks) chunk_pair_planes(E, L.maxkeys);

  // ---- records (interior / keep flags for the backward), frame-bucket counts and touched-tile masks;
  //      scores start at 0
  const uint64_t qglob = ((static_cast<uint64_t>(T.b) * P.T + T.tg) * P.H + qh) * P.W + qw;
  for (int s = 0; s < jper; ++s) {
    const int j = js + s;
    int bk = -1, pa = -1, pb = -1;
    uint32_t bits = 0u;
    if (qvalid && s < n) {
      const unsigned long long raw = S.rec[qbase + j];
      const float pt = __uint_as_float(static_cast<uint32_t>(raw)), ph = __uint_as_float(static_cast<uint32_t>(raw >> 32));
      const float pw = sacc[j];
      sacc[j] = 0.f;
      const int t0 = static_cast<int>(floorf(pt)), h0 = static_cast<int>(floorf(ph)), w0 = static_cast<int>(floorf(pw));
      unsigned long long v = 0ull;
      if (work && t0 + 1 >= E.zlo && t0 <= E.zhi) {  // a corner in a frame the K/V buffers hold
        const int dz = t0 - E.zlo + 1;
        const bool keep = !P.drop_thresh ||
                          dropout_keep(P.seed, (qglob * P.nh + T.head) * static_cast<uint64_t>(KG) + j, P.drop_thresh);
        v = pack_rec(pt - static_cast<float>(t0), ph - static_cast<float>(h0), pw - static_cast<float>(w0), dz,
                     h0 - E.ylo, w0 - E.xlo) |
            (clip_grad_mult(pt, P.T) != 0.f ? 1ull << kBitInT : 0ull) |
            (clip_grad_mult(ph, P.H) != 0.f ? 1ull << kBitInH : 0ull) |
            (clip_grad_mult(pw, P.W) != 0.f ? 1ull << kBitInW : 0ull) | (keep ? 1ull << kBitKeep : 0ull);
        bk = dz;
        if (masks) {
          const int iy = axis_chunk_of(h0, E.ylo, E.R, E.ny), ix = axis_chunk_of(w0, E.xlo, E.cw, E.nx);
          const int ya = E.ylo + iy * (E.R - 1), xa = E.xlo + ix * (E.cw - 1);
          bits = corner_tiles((h0 - ya) * E.kst + (w0 - xa), E.kst, w0 + 1 < P.W, h0 + 1 < P.H);
          const int chk = iy * E.nx + ix;
          if (t0 >= E.zlo) pa = dz * kMaxMaskChunks + chk;
          if (t0 + 1 <= E.zhi) pb = (dz + 1) * kMaxMaskChunks + chk;
          v |= static_cast<unsigned long long>(chk) << kBitChunk;
          bk += chk * 32;
        }
      }
      S.rec[qbase + j] = v;
    }
    if (bk >= 0) atomicAdd(S.bcur + bk, 1);  // plain shared atomics: faster than warp-matched ones here
    if (pa >= 0 && (S.mask[pa] & bits) != bits) atomicOr(S.mask + pa, bits);
    if (pb >= 0 && (S.mask[pb] & bits) != bits) atomicOr(S.mask + pb, bits);
  }
  if (qvalid)
    for (int e = K + sub; e < KG; e += kLPQ) sacc[e] = 0.f;
  __syncthreads();
  if (warp == 0) scan_buckets(S.bcur, S.bstart);
  if (P.saved) {  // the records and the raw envelope for the tensor-core backward
    if (qvalid) {
      unsigned long long* dst = static_cast<unsigned long long*>(P.saved) +
                                ((static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow) * K;
      for (int j = sub; j < K; j += kLPQ) dst[j] = S.rec[qbase + j];
    }
    if (threadIdx.x == 32) {
      int4* env = reinterpret_cast<int4*>(static_cast<char*>(P.saved) + saved_env_offset(P)) + 2 * blockIdx.x;
      env[0] = make_int4(S.env[0], S.env[1], S.env[2], S.env[3]);
      env[1] = make_int4(S.env[4], S.env[5], 0, 0);
    }
  }
  __syncthreads();
  if (overflow) {  // the records cannot encode this envelope: the CUDA-core gather computes the tile
    tile_fallback<DCH, false>(P, T);
    return;  // no copy was issued yet
  }
  for (int s = 0; s < jper; ++s) {  // hit list: every active sample once, grouped by (chunk, frame) bucket
    const int j = js + s;
    int bk = -1;
    if (qvalid && s < n) {
      const unsigned long long v = S.rec[qbase + j];
      if (v >> 63) bk = rec_bucket(v);
    }
    if (bk >= 0) S.hits[atomicAdd(S.bcur + bk, 1)] = static_cast<unsigned short>(qbase + j);
  }
  const int g = lane >> 2, t4 = lane & 3;
  float* grow_s = S.sbuf + static_cast<size_t>(r) * 16 * L.sld;  // the row group's 16 dense rows
  const __nv_bfloat16* qgrp = S.qs + static_cast<size_t>(r) * 16 * L.rs;
  __syncthreads();

  // ---- pass 1: scores (hits CTA-wide); the next chunk's keys load while this chunk's samples combine
  const int nz = work ? E.zhi - E.zlo + 1 : 0;
  const __nv_bfloat16* kg = static_cast<const __nv_bfloat16*>(P.k);
  const __nv_bfloat16* vg = static_cast<const __nv_bfloat16*>(P.v);
  const int kst = E.kst;
  {
    Chunk k;
    bool have = chunk_first(E, S.mask, masks, nz, k);
    if (have) {
      if (tma) {
        if (!*S.dead) issue_keys_tma(P, T, E, k, S.kbuf, L.rs, maps.k, maps.have, kbar, true);
      } else {
        issue_keys<DCH>(P, T, E, k, S.kbuf, L.rs, kg, P.k_ld);
      }
    }
    while (have) {
      const Chunk cur = k;
      if (tma) {
        wait_keys(kbar, kphase, S.dead, P.status);
        kphase ^= 1u;
      } else {
        cp_async_wait_all();
      }
      __syncthreads();
      if (tma && tile_dead(S.dead)) break;  // a wait gave up: nothing more reads the key buffer
      dense_tiles<DCH, kWPG>(S.kbuf, qgrp, L.rs, grow_s, L.sld, part, cur.m);
      __syncthreads();
      have = chunk_next(E, S.mask, masks, nz, k);
      if (have) {
        if (tma) {
          if (!*S.dead) issue_keys_tma(P, T, E, k, S.kbuf, L.rs, maps.k, maps.have, kbar, false);
        } else {
          issue_keys<DCH>(P, T, E, k, S.kbuf, L.rs, kg, P.k_ld);
        }
      }
      const int zb = E.zlo + cur.zr * E.pg, ya = chunk_ya(E, cur), xa = chunk_xa(E, cur);
      // hits with a corner in the chunk's planes: buckets t0 - zlo + 1 = zb - zlo .. zb - zlo + pg
      const int hb = (masks ? cur.iy * E.nx + cur.ix : 0) * 32 + cur.zr * E.pg;
      const int hlo = S.bstart[hb], hhi = S.bstart[hb + E.pg + 1];
      for (int i = hlo + static_cast<int>(threadIdx.x); i < hhi; i += kThreads) {
        const int idx = S.hits[i];
        const int q = static_cast<int>((static_cast<float>(idx) + 0.5f) * invK);
        const Rec rc = decode_rec(S.rec[idx], E);
        if (fsplit && (axis_chunk_of(rc.h0, E.ylo, E.R, E.ny) != cur.iy || axis_chunk_of(rc.w0, E.xlo, E.cw, E.nx) != cur.ix))
          continue;
        const float* row = S.sbuf + static_cast<size_t>(q) * L.sld + (rc.h0 - ya) * kst + (rc.w0 - xa);
        float* sp = S.sacc + static_cast<size_t>(q) * KG + (idx - q * K);
        const int pa = rc.t0 - zb;  // chunk plane of the lower corner: -1 .. pg - 1
        if (pa >= 0) *sp = fmaf(frac_weight(rc.ft, false), plane_bil(row + pa * E.kpp, kst, rc, P.H, P.W), *sp);
        if (pa + 1 < E.pg)
          *sp = fmaf(frac_weight(rc.ft, true), plane_bil(row + (pa + 1) * E.kpp, kst, rc, P.H, P.W), *sp);
      }
    }
  }

  // ---- extra keys: S_extra = Q . EK^T (all G keys in one chunk of the key buffer)
  const int gp = (P.G + 15) & ~15;
  const uint32_t gmask = gp >= 512 ? 0xffffffffu : (1u << (gp >> 4)) - 1u;
  if (P.G > 0) {
    __syncthreads();
    load_extra<DCH>(P, T, S.kbuf, L.rs, P.ek, gp);
    __syncthreads();
    dense_tiles<DCH, kWPG>(S.kbuf, qgrp, L.rs, grow_s, L.sld, part, gmask);
    __syncthreads();
    if (qvalid)
      for (int e = sub; e < P.G; e += kLPQ) sacc[K + e] = S.sbuf[static_cast<size_t>(qi) * L.sld + e];
  }
  __syncthreads();

  // ---- softmax over the K (+G) scores of each query; optional saved probabilities; P~ row scales
  float m = -INFINITY;
  if (qvalid)
    for (int j = sub; j < KG; j += kLPQ) m = fmaxf(m, sacc[j] * P.scale_log2);
#pragma unroll
  for (int o = 1; o < kLPQ; o <<= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
  float l = 0.f;
  if (qvalid)
    for (int j = sub; j < KG; j += kLPQ) l += exp2f(sacc[j] * P.scale_log2 - m);
#pragma unroll
  for (int o = 1; o < kLPQ; o <<= 1) l += __shfl_xor_sync(kFull, l, o);
  float bp = 0.f;
  if (qvalid) {
    float* prob_row = P.probs ? P.probs + ((static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow) * K : nullptr;
    const float inv_l = 1.f / l;
    const uint64_t qg = ((static_cast<uint64_t>(T.b) * P.T + T.tg) * P.H + qh) * P.W + qw;
    for (int j = sub; j < KG; j += kLPQ) {
      const float p = exp2f(sacc[j] * P.scale_log2 - m);
      if (prob_row && j < K) prob_row[j] = p * inv_l;
      float pv = p;
      if (P.drop_thresh)
        pv = dropout_keep(P.seed, (qg * P.nh + T.head) * static_cast<uint64_t>(KG) + j, P.drop_thresh)
                 ? p * P.drop_keep_scale : 0.f;
      sacc[j] = pv;  // unnormalised, dropout applied
      bp += pv;
    }
  }
#pragma unroll
  for (int o = 1; o < kLPQ; o <<= 1) bp += __shfl_xor_sync(kFull, bp, o);
  if (sub == 0) {
    S.lrow[qi] = l;
    S.qsc[qi] = bp > 0.f ? kFixRange / bp : 1.f;
    S.qsc[kQ + qi] = bp > 0.f ? bp / kFixRange : 0.f;
    if (qvalid) P.lse[(static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow] = m + log2f(l);
  }
  __syncthreads();

  // ---- pass 2: O = P~ . V (hits CTA-wide)
  // the 8 warps of a row group: kCG channel ranges (sizes differ by at most one tile) x kKS parts of the
  // touched tiles (every kKS-th one): a P~ fragment and a V tile are read once per row group for
  // head_dim <= 72 (all channel tiles per warp; measured faster than 2 or 4 ranges), the parts' partial
  // sums are added once at the end
  constexpr int kCG = pv_channel_groups(DCH), kKS = kWPG / kCG;
  constexpr int kCB = DCH / kCG, kCX = DCH % kCG;
  constexpr int kTPW = kCB + (kCX ? 1 : 0);  // channel tiles per warp (at most)
  const int cpart = part % kCG, kpar = part / kCG;
  const int nt0 = cpart * kCB + min(cpart, kCX), nt1 = nt0 + kCB + (cpart < kCX ? 1 : 0);
  float o[kTPW + 1][4];
#pragma unroll
  for (int i = 0; i < kTPW + 1; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const __nv_bfloat16* tp = reinterpret_cast<const __nv_bfloat16*>(S.sbuf);  // P~^T after the transposition
  {
    Chunk k;
    for (bool have = chunk_first(E, S.mask, masks, nz, k); have; have = chunk_next(E, S.mask, masks, nz, k)) {
      __syncthreads();  // the previous chunk's product is done with the key buffer and the dense tile
      zero_tiles<kQ>(S.sbuf, L.sld, k.m);
      const int zb = E.zlo + k.zr * E.pg, ya = chunk_ya(E, k), xa = chunk_xa(E, k);
      const int hb = (masks ? k.iy * E.nx + k.ix : 0) * 32 + k.zr * E.pg;
      const int hlo = S.bstart[hb], hhi = S.bstart[hb + E.pg + 1];
      __syncthreads();
      // the values land while the weights are scattered and converted (issued here, not in the short
      // zeroing phase above: the issuing warps have the fewest hits below)
      if (tma) {
        if (!*S.dead) issue_keys_tma(P, T, E, k, S.kbuf, L.rs, maps.v, maps.have, kbar, P.G > 0);
      } else {
        issue_keys<DCH>(P, T, E, k, S.kbuf, L.rs, vg, P.v_ld);
      }
      for (int i = hlo + static_cast<int>(threadIdx.x); i < hhi; i += kThreads) {
        const int idx = S.hits[i];
        const int q = static_cast<int>((static_cast<float>(idx) + 0.5f) * invK);
        const float pv = S.sacc[static_cast<size_t>(q) * KG + (idx - q * K)];
        if (pv == 0.f) continue;
        const Rec rc = decode_rec(S.rec[idx], E);
        if (fsplit && (axis_chunk_of(rc.h0, E.ylo, E.R, E.ny) != k.iy || axis_chunk_of(rc.w0, E.xlo, E.cw, E.nx) != k.ix))
          continue;
        int* row = reinterpret_cast<int*>(S.sbuf) + static_cast<size_t>(q) * L.sld;
        const int k00 = (rc.h0 - ya) * kst + (rc.w0 - xa);
        const float ps = pv * S.qsc[q];
        const int pa = rc.t0 - zb;  // chunk plane of the lower corner: -1 .. pg - 1
        if (pa >= 0) scatter_fixed_row(row + pa * E.kpp, k00, kst, rc, ps * frac_weight(rc.ft, false), P.H, P.W);
        if (pa + 1 < E.pg)
          scatter_fixed_row(row + (pa + 1) * E.kpp, k00, kst, rc, ps * frac_weight(rc.ft, true), P.H, P.W);
      }
      __syncthreads();
      transpose_fixed<kMaxKeysFwd>(S.sbuf, L.sld, k.m, S.qsc + kQ);
      if (tma) {
        wait_keys(kbar, kphase, S.dead, P.status);
        kphase ^= 1u;
      } else {
        cp_async_wait_all();
      }
      __syncthreads();
      if (tma && tile_dead(S.dead)) break;  // a wait gave up: nothing more reads the key buffer
      dq_product<DCH, kTPW, kKS>(tp, r, S.kbuf, L.rs, nt0, nt1, k.m, o, kpar);
    }
  }
  if (P.G > 0) {  // extra values: their weights straight into the fixed-point rows
    __syncthreads();
    load_extra<DCH>(P, T, S.kbuf, L.rs, P.ev, gp);
    zero_tiles<kQ>(S.sbuf, L.sld, gmask);
    __syncthreads();
    if (qvalid)
      for (int e = sub; e < P.G; e += kLPQ)
        reinterpret_cast<int*>(S.sbuf)[static_cast<size_t>(qi) * L.sld + e] = fix_round(sacc[K + e] * S.qsc[qi]);
    __syncthreads();
    transpose_fixed<kMaxKeysFwd>(S.sbuf, L.sld, gmask, S.qsc + kQ);
    __syncthreads();
    dq_product<DCH, kTPW, kKS>(tp, r, S.kbuf, L.rs, nt0, nt1, gmask, o, kpar);
  }

  // ---- the warps of the other key-tile parts hand their partial sums to part 0 (through the key
  //      buffer and the dense tile, contiguous and free now: [2][kCG][kKS - 1][kTPW][32] float4)
  if (kKS > 1) {
    __syncthreads();  // every product is done with the key buffer and the dense tile
    float4* red = reinterpret_cast<float4*>(S.kbuf) + ((r * kCG + cpart) * (kKS - 1) * kTPW) * 32 + lane;
    if (kpar > 0) {
#pragma unroll
      for (int j = 0; j < kTPW; ++j)
        if (nt0 + j < nt1) red[((kpar - 1) * kTPW + j) * 32] = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
    }
    __syncthreads();
    if (kpar == 0) {
      for (int u = 0; u < kKS - 1; ++u) {
#pragma unroll
        for (int j = 0; j < kTPW; ++j) {
          if (nt0 + j >= nt1) continue;
          const float4 t = red[(u * kTPW + j) * 32];
          o[j][0] += t.x;
          o[j][1] += t.y;
          o[j][2] += t.z;
          o[j][3] += t.w;
        }
      }
    }
  }

  // ---- normalise and store (first-half warps)
  if (kpar == 0) {
    int qh0_, qw0_, qh1_, qw1_;
    query_hw(T, r, g, qh0_, qw0_);
    query_hw(T, r, g + 8, qh1_, qw1_);
    const bool v0 = qh0_ < P.H && qw0_ < P.W, v1 = qh1_ < P.H && qw1_ < P.W;
    const float inv0 = v0 ? 1.f / S.lrow[r * 16 + g] : 0.f;
    const float inv1 = v1 ? 1.f / S.lrow[r * 16 + g + 8] : 0.f;
    __nv_bfloat16* o0 = static_cast<__nv_bfloat16*>(P.out) +
        (static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + qh0_) * P.W + qw0_) * P.out_ld + T.head * P.d;
    __nv_bfloat16* o1 = static_cast<__nv_bfloat16*>(P.out) +
        (static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + qh1_) * P.W + qw1_) * P.out_ld + T.head * P.d;
#pragma unroll
    for (int j = 0; j < kTPW; ++j) {
      const int nt = nt0 + j;
      if (nt >= nt1) continue;
      if (v0) *reinterpret_cast<__nv_bfloat162*>(o0 + nt * 8 + 2 * t4) = __floats2bfloat162_rn(o[j][0] * inv0, o[j][1] * inv0);
      if (v1) *reinterpret_cast<__nv_bfloat162*>(o1 + nt * 8 + 2 * t4) = __floats2bfloat162_rn(o[j][2] * inv1, o[j][3] * inv1);
    }
  }
}

}  // namespace fwd
}  // namespace tc

// ------------------------------------------------------------------------------ host side
long long saved_bytes(const AttnParams& P) {
  const long long tiles = static_cast<long long>(P.B) * P.q_frames * ((P.H + tc::t32::kTileH - 1) / tc::t32::kTileH) *
                          ((P.W + tc::kTileW - 1) / tc::kTileW) * P.nh;
  return saved_env_offset(P) + tiles * 32;
}

bool tc_supported(const AttnParams& P) {
  if (P.dtype != MSL_DTYPE_BF16) return false;
  if (P.d % 8 != 0 || P.d < 16 || P.d > 128) return false;
  if (P.T > 65535 || P.K > 2048 || P.G > 256) return false;
  if (static_cast<long long>(P.kv_frames) * P.H * P.W > 0x7fffffffLL) return false;  // 32-bit key rows
  if (static_cast<long long>(tc::t32::kQ) * P.K > 65536) return false;  // hit-list entries are 16-bit
  // base-grid tables hold at most 96 positions per axis
  if (P.kt > 96 || P.kh + tc::t32::kTileH - 1 > 96 || P.kw + tc::kTileW - 1 > 96) return false;
  return true;
}

bool tc_plan(const AttnParams& P, TcLaunch& L, int smem_limit) {
  const int dch = P.d / 8;
  L.rs = (dch & 1) ? P.d : P.d + 8;  // odd number of 16-byte chunks per row: conflict-free ldmatrix
  L.tiles_h = (P.H + tc::t32::kTileH - 1) / tc::t32::kTileH;
  L.tiles_w = (P.W + tc::kTileW - 1) / tc::kTileW;
  const size_t fixed = tc::fwd::smem_fixed(P, L.rs);
  const size_t per_key = static_cast<size_t>(L.rs) * 2 + static_cast<size_t>(tc::t32::kQ) * 4;
  const size_t slack = static_cast<size_t>(tc::t32::kQ) * 8 * 4;  // dense-row padding (sld = maxkeys + 8)
  if (fixed + slack + per_key * 64 > static_cast<size_t>(smem_limit)) return false;
  int mk = static_cast<int>((static_cast<size_t>(smem_limit) - fixed - slack) / per_key);
  mk &= ~15;
  const int gp = (P.G + 15) & ~15;
  if (mk < 64) return false;
  if (mk > tc::t32::kMaxKeysFwd) mk = tc::t32::kMaxKeysFwd;
  if (mk < gp) return false;
  L.maxkeys = mk;
  L.sld = mk + 8;  // row stride = 8 or 24 (mod 32) words: mma fragment rows hit distinct banks
  // a transposed bf16 tile [maxkeys][40] must fit in the dense fp32 tile [32][sld]
  if (static_cast<size_t>(mk) * tc::t32::kTRow * 2 > static_cast<size_t>(tc::t32::kQ) * L.sld * 4) return false;
  // the output partial sums handed between the warps of a row group fit the key buffer + dense tile
  {
    const int cg = tc::fwd::pv_channel_groups(dch), ks = tc::t32::kWPG / cg;
    const int tpw = (dch + cg - 1) / cg;
    if (static_cast<size_t>(2) * cg * (ks - 1) * tpw * 512 >
        static_cast<size_t>(mk) * L.rs * 2 + static_cast<size_t>(tc::t32::kQ) * L.sld * 4)
      return false;
  }
  // the setup stages 32 queries x K x 3 offsets (rows padded to 16 bytes) and the head's K x 3 offset
  // bias in the key buffer + the dense tile
  if (static_cast<size_t>(mk) * L.rs * 2 + static_cast<size_t>(tc::t32::kQ) * L.sld * 4 <
      (static_cast<size_t>(tc::t32::kQ) * ((3 * P.K + 6) & ~3) + 3 * P.K) * 4)
    return false;
  L.smem = static_cast<size_t>(mk) * L.rs * 2 + static_cast<size_t>(tc::t32::kQ) * L.sld * 4 + fixed;
  L.tiles = static_cast<long long>(P.B) * P.q_frames * L.tiles_h * L.tiles_w * P.nh;
  return L.tiles <= 0x7fffffffLL && L.smem <= static_cast<size_t>(smem_limit);
}

template <int DCH>
static cudaError_t launch_fwd_tc_t(const AttnParams& P, const TcLaunch& L, const tc::KeyMaps& maps,
                                   cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(tc::fwd::dsa_fwd_tc_kernel<DCH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  tc::fwd::dsa_fwd_tc_kernel<DCH><<<static_cast<unsigned>(L.tiles), tc::kThreads, L.smem, s>>>(P, L, maps);
  return cudaGetLastError();
}

namespace tc {

// One tensor map over head-sliced [B, Nkv, ld] bf16 rows: dims (channel, x, y, frame, sample), box
// (rs channels, bw columns, 1, 1, 1), zero fill outside.
static bool make_key_map(CUtensorMap* map, const AttnParams& P, const void* base, long long ld, int rs, int bw,
                         int bh) {
  using Encode = PFN_cuTensorMapEncodeTiled_v12000;
  static const Encode encode = []() -> Encode {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<Encode>(fn);
  }();
  if (!encode || !base) return false;
  // 16-byte aligned base and row stride; the box within the tensor's extents
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 2) & 15) || (rs * 2) % 16 != 0 || rs > 256) return false;
  if (static_cast<long long>(P.nh) * P.d < rs || P.W < bw || P.H < bh || ld < static_cast<long long>(P.nh) * P.d)
    return false;
  const cuuint64_t dims[5] = {static_cast<cuuint64_t>(P.nh) * P.d, static_cast<cuuint64_t>(P.W),
                              static_cast<cuuint64_t>(P.H), static_cast<cuuint64_t>(P.kv_frames),
                              static_cast<cuuint64_t>(P.B)};
  const cuuint64_t row = static_cast<cuuint64_t>(ld) * 2;
  const cuuint64_t strides[4] = {row, row * P.W, row * P.W * P.H, row * static_cast<cuuint64_t>(P.Nkv)};
  const cuuint32_t box[5] = {static_cast<cuuint32_t>(rs), static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh), 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  if (strides[3] >= (1ull << 40)) return false;
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_key_maps(KeyMaps* maps, const AttnParams& P, int rs) {
  memset(maps, 0, sizeof(*maps));
  // MSL_TC_LOADS=cpasync selects the cp.async loads (both paths compute the same results)
  const char* sel = getenv("MSL_TC_LOADS");
  if (sel && strcmp(sel, "cpasync") == 0) return false;
  for (int j = 0; j < 4; ++j)
    for (int h = 0; h < 4; ++h)
      if (make_key_map(&maps->k[j][h], P, P.k, P.k_ld, rs, 8 * (j + 1), 1 << h) &&
          make_key_map(&maps->v[j][h], P, P.v, P.v_ld, rs, 8 * (j + 1), 1 << h))
        maps->have |= 1 << (4 * j + h);
  // test hook for the bounded TMA wait: MSL_TEST_TMA_NO_COPY=1 arms every chunk's byte count but issues
  // no copy, so each CTA's first wait runs out (about a second) and sets MSL_STATUS_TIMEOUT
  const char* nocopy = getenv("MSL_TEST_TMA_NO_COPY");
  if (nocopy && strcmp(nocopy, "1") == 0 && (maps->have & 1)) maps->have |= static_cast<int>(0x80000000u);
  return maps->have & 1;  // the one-row 8-column boxes serve every chunk width
}

}  // namespace tc

cudaError_t launch_attn_fwd_tc(const AttnParams& P, const TcLaunch& L0, cudaStream_t s) {
  TcLaunch L = L0;
  tc::KeyMaps maps;
  L.tma = tc::make_key_maps(&maps, P, L.rs);
  switch (P.d / 8) {
    case 2: return launch_fwd_tc_t<2>(P, L, maps, s);
    case 3: return launch_fwd_tc_t<3>(P, L, maps, s);
    case 4: return launch_fwd_tc_t<4>(P, L, maps, s);
    case 5: return launch_fwd_tc_t<5>(P, L, maps, s);
    case 6: return launch_fwd_tc_t<6>(P, L, maps, s);
    case 7: return launch_fwd_tc_t<7>(P, L, maps, s);
    case 8: return launch_fwd_tc_t<8>(P, L, maps, s);
    case 9: return launch_fwd_tc_t<9>(P, L, maps, s);
    case 10: return launch_fwd_tc_t<10>(P, L, maps, s);
    case 11: return launch_fwd_tc_t<11>(P, L, maps, s);
    case 12: return launch_fwd_tc_t<12>(P, L, maps, s);
    case 13: return launch_fwd_tc_t<13>(P, L, maps, s);
    case 14: return launch_fwd_tc_t<14>(P, L, maps, s);
    case 15: return launch_fwd_tc_t<15>(P, L, maps, s);
    case 16: return launch_fwd_tc_t<16>(P, L, maps, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace msl
