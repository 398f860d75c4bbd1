// Tensor-core ("key envelope") formulation of the deformable gather attention forward, bf16.
//
// One CTA owns a tile of 8 x 8 queries of one frame, one head and one sample (64 queries, 16 warps:
// four per 16-query row group; 8 lanes per query share its per-sample work).
// Every trilinear corner any of the tile's 64 x K samples can touch lies in the tile's key
// envelope: frames [zlo, zhi] x rows [ylo, yhi] x columns [xlo, xhi].  The CTA walks that
// envelope one frame ("plane") at a time, in chunks of at most `maxkeys` keys (rows and columns
// split with a one-row / one-column overlap so that the four corners a sample has in a plane
// always fall in one chunk):
//
//   pass 1, per chunk:  S = Q . K_chunk^T on the tensor cores (mma.sync m16n8k16 bf16 -> fp32,
//                       one 16-query row group per warp pair), kept in shared memory; every sample
//                       with corners in the chunk adds  sum_corners w_c * S[q, corner]  to its score.
//   softmax:            per query over its K samples (+ G extra keys, scored the same way).
//   pass 2, per chunk:  every sample scatters p * w_c into a dense P~[q, key] (shared memory), then
//                       O += P~ . V_chunk on the tensor cores (ldmatrix.trans for V).
//
// The dense products are redundant (the envelope holds more keys than the samples' corners), but
// they run on the tensor cores and replace 8 * d scalar FMAs and 8 gathered d-vectors per sample
// by 8 shared-memory reads of scalars.  Sample coordinates come from the offsets with the same float32
// arithmetic as the CUDA-core kernels (msl_common.cuh), so corner choices are identical; each sample's
// corner and trilinear fractions are computed once per tile and kept as a packed 8-byte record
// (fractions quantised to 12 bits: interpolation weights within 1.2e-4 - this path is bf16 only).
// Reference semantics: infinity/video/attention.py:113-186 (grid, grid_sample, softmax, dropout,
// value sum) and :159-173 (extra keys).

#include "dsa_tc.cuh"

namespace msl {
namespace tc {

constexpr int kWPG = kWarps / 4;      // warps per 16-query row group
constexpr int kLPQ = kWPG * 32 / 16;  // lanes per query for the per-sample work
constexpr int kTileH = 8, kQ = kTileH * kTileW;

// Shared-memory layout, sized by the host (TcLaunch).
struct Smem {
  __nv_bfloat16* kbuf;  // [maxkeys][rs]
  float* sbuf;          // [4][16][sld]
  float* sacc;          // [64][K + G]
  unsigned long long* rec;  // [64][K] packed sample records (see pack_rec)
  int* env;             // [16] envelope, then base-grid tables (float) from env + 16
  float* mrow;          // [64]
  float* lrow;          // [64]
};

__device__ __forceinline__ Smem carve(unsigned char* base, const AttnParams& P, const TcLaunch& L) {
  Smem s;
  size_t off = 0;
  s.kbuf = reinterpret_cast<__nv_bfloat16*>(base + off);
  off += static_cast<size_t>(L.maxkeys) * L.rs * 2;
  s.sbuf = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(4) * 16 * L.sld * 4;
  s.rec = reinterpret_cast<unsigned long long*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 8;
  s.sacc = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * (P.K + P.G) * 4;
  s.env = reinterpret_cast<int*>(base + off);
  off += kEnvWords * 4;
  s.mrow = reinterpret_cast<float*>(base + off);
  off += kQ * 4;
  s.lrow = reinterpret_cast<float*>(base + off);
  return s;
}

template <int DCH>
__global__ void __launch_bounds__(kThreads, 1) dsa_fwd_tc_kernel(const AttnParams P, const TcLaunch L) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const Smem S = carve(smem_raw, P, L);
  const TileCtx T = decode_tile(P, L, kTileH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp / kWPG, part = warp - (warp / kWPG) * kWPG;
  const int ll = part * 32 + lane;           // 0..127 within the row group
  const int cq = ll / kLPQ, sub = ll - (ll / kLPQ) * kLPQ;  // owned query (0..15) and lane of that query
  const int K = P.K, KG = P.K + P.G;
  // the kLPQ lanes of a query own contiguous window ranges, so a lane's samples touch few frames and
  // whole lanes skip the frames they cannot reach
  const int jper = (K + kLPQ - 1) / kLPQ;
  const int js = min(K, sub * jper), je = min(K, js + jper);
  const SampleGeom sg{P.T, P.H, P.W, P.kt, P.kh, P.kw, P.oscale};

  int qh, qw;
  query_hw(T, r, cq, qh, qw);
  const bool qvalid = qh < P.H && qw < P.W;
  const long long qrow = (static_cast<long long>(T.tl) * P.H + qh) * P.W + qw;
  const float* orow = P.offsets + (static_cast<long long>(T.b) * P.Nq + qrow) * P.off_ld +
                      static_cast<long long>(T.head) * K * 3;
  float* sacc = S.sacc + static_cast<size_t>(r * 16 + cq) * KG;
  unsigned long long* rec = S.rec + static_cast<size_t>(r * 16 + cq) * K;

  float* tabz = reinterpret_cast<float*>(S.env + 16);
  float* taby = tabz + 96;
  float* tabx = taby + 96;
  if (threadIdx.x == 0) {
    S.env[0] = 0x7fffffff; S.env[1] = -0x7fffffff; S.env[2] = 0x7fffffff;
    S.env[3] = -0x7fffffff; S.env[4] = 0x7fffffff; S.env[5] = -0x7fffffff;
  }
  fill_tabs(P, T, kTileH, tabz, taby, tabx);
  __syncthreads();
  const Tabs tb{tabz, taby, tabx};
  const int qy = qh - T.qh0, qx = qw - T.qw0;

  // ---- setup: sample coordinates.  This head's offsets of the tile are staged in the key / score
  // buffers (unused until pass 1) with one wave of cp.async per round of 32 queries (row groups 0-1,
  // then 2-3), so the coordinate pass reads shared memory instead of a dependent global round trip
  // per sample.  Raw coordinates are kept in rec / sacc until the envelope is known.
  const int K3 = 3 * K;
  float* ostage = reinterpret_cast<float*>(S.kbuf);
  const int kvlo = max(P.kv_frame0, 0), kvhi = min(P.kv_frame0 + P.kv_frames, P.T) - 1;
  int zmn = 0x7fffffff, zmx = -0x7fffffff, ymn = 0x7fffffff, ymx = -0x7fffffff, xmn = 0x7fffffff, xmx = -0x7fffffff;
  bool miss = false;
  for (int round = 0; round < 2; ++round) {
    __syncthreads();
    for (int qi = round * 32 + warp; qi < round * 32 + 32; qi += kWarps) {
      int sqh, sqw;
      query_hw(T, qi >> 4, qi & 15, sqh, sqw);
      if (sqh >= P.H || sqw >= P.W) continue;
      const float* src = P.offsets +
                         (static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + sqh) * P.W + sqw) * P.off_ld +
                         static_cast<long long>(T.head) * K3;
      float* dst = ostage + static_cast<size_t>(qi - round * 32) * K3;
      for (int k = lane; k < K3; k += 32) cp_async4(smem_u32(dst + k), src + k);
    }
    cp_async_wait_all();
    __syncthreads();
    if ((r >> 1) != round) continue;
    const float* oq = ostage + static_cast<size_t>(r * 16 + cq - round * 32) * K3;
    WinIdx wi;
    wi.init(js, P.kh, P.kw);
#pragma unroll 2
    for (int j = js; j < je; ++j, wi.advance(1, P.kh, P.kw)) {
      if (!qvalid) {
        rec[j] = 0ull;
        sacc[j] = 0.f;
        continue;
      }
      float pt, ph, pw;
      tab_coords(P, tb, qy, qx, wi.it, wi.ih, wi.iw, oq[3 * j], oq[3 * j + 1], oq[3 * j + 2], pt, ph, pw);
      rec[j] = (static_cast<unsigned long long>(__float_as_uint(ph)) << 32) | __float_as_uint(pt);
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
  for (int j = K + sub; j < KG; j += kLPQ) sacc[j] = 0.f;
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
    const int nxk = E.xhi - E.xlo + 1;
    E.cw = nxk <= L.maxkeys / 2 ? nxk : L.maxkeys / 2;
    E.R = L.maxkeys / E.cw;
    E.ny = axis_chunks(E.ylo, E.yhi, E.R);
    E.nx = axis_chunks(E.xlo, E.xhi, E.cw);
  } else {
    E.cw = E.R = E.ny = E.nx = 1;
  }
  const bool split = E.ny * E.nx > 1;
  // records hold t0 - zlo + 1 in 5 bits and h0 - ylo, w0 - xlo in 8 bits
  const bool chunk_overflow = any && (E.zhi - E.zlo + 2 > 31 || E.yhi - E.ylo > 255 || E.xhi - E.xlo > 255);
  if (chunk_overflow && threadIdx.x == 0 && P.status) atomicOr(P.status, MSL_STATUS_TC_RANGE);

  // pack the per-sample records now that the envelope is known; the lane's frame range [zl_lo, zl_hi]
  // (relative, as zrel) bounds the frames its samples touch
  int zl_lo = 0x7fff, zl_hi = -1;
  for (int j = js; j < je; ++j) {
    if (!qvalid) continue;
    const unsigned long long raw = rec[j];
    const float pt = __uint_as_float(static_cast<uint32_t>(raw)), ph = __uint_as_float(static_cast<uint32_t>(raw >> 32));
    const float pw = sacc[j];
    sacc[j] = 0.f;
    const int t0 = static_cast<int>(floorf(pt)), h0 = static_cast<int>(floorf(ph)), w0 = static_cast<int>(floorf(pw));
    if (!any || chunk_overflow || t0 + 1 < E.zlo || t0 > E.zhi) {  // no corner in a frame the K/V buffers hold
      rec[j] = 0ull;
      continue;
    }
    rec[j] = pack_rec(pt - static_cast<float>(t0), ph - static_cast<float>(h0), pw - static_cast<float>(w0),
                      t0 - E.zlo + 1, h0 - E.ylo, w0 - E.xlo);
    zl_lo = min(zl_lo, t0 - E.zlo + 1);
    zl_hi = max(zl_hi, t0 - E.zlo + 2);
  }

  // ---- Q fragments (rows g and g + 8 of the group)
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t qa[DCH / 2 > 0 ? DCH / 2 : 1][4];
  uint32_t qt[2] = {0u, 0u};
  {
    int qh0_, qw0_, qh1_, qw1_;
    query_hw(T, r, g, qh0_, qw0_);
    query_hw(T, r, g + 8, qh1_, qw1_);
    const bool v0 = qh0_ < P.H && qw0_ < P.W, v1 = qh1_ < P.H && qw1_ < P.W;
    const __nv_bfloat16* q0 = static_cast<const __nv_bfloat16*>(P.q) +
        (static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + qh0_) * P.W + qw0_) * P.q_ld + T.head * P.d;
    const __nv_bfloat16* q1 = static_cast<const __nv_bfloat16*>(P.q) +
        (static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + qh1_) * P.W + qw1_) * P.q_ld + T.head * P.d;
#pragma unroll
    for (int ks = 0; ks < DCH / 2; ++ks) {
      qa[ks][0] = v0 ? __ldg(reinterpret_cast<const unsigned int*>(q0 + ks * 16 + 2 * t4)) : 0u;
      qa[ks][1] = v1 ? __ldg(reinterpret_cast<const unsigned int*>(q1 + ks * 16 + 2 * t4)) : 0u;
      qa[ks][2] = v0 ? __ldg(reinterpret_cast<const unsigned int*>(q0 + ks * 16 + 8 + 2 * t4)) : 0u;
      qa[ks][3] = v1 ? __ldg(reinterpret_cast<const unsigned int*>(q1 + ks * 16 + 8 + 2 * t4)) : 0u;
    }
    if constexpr (DCH & 1) {
      qt[0] = v0 ? __ldg(reinterpret_cast<const unsigned int*>(q0 + (DCH - 1) * 8 + 2 * t4)) : 0u;
      qt[1] = v1 ? __ldg(reinterpret_cast<const unsigned int*>(q1 + (DCH - 1) * 8 + 2 * t4)) : 0u;
    }
  }
  const float* srow_q = S.sbuf + (static_cast<size_t>(r) * 16 + cq) * L.sld;  // scores of the owned query

  // ---- pass 1: scores
  if (any && !chunk_overflow) {
    for (int z = E.zlo; z <= E.zhi; ++z) {
      const int zrel = z - E.zlo + 1;
      for (int iy = 0; iy < E.ny; ++iy) {
        const int ya = E.ylo + iy * (E.R - 1), yb = min(ya + E.R - 1, E.yhi);
        for (int ix = 0; ix < E.nx; ++ix) {
          const int xa = E.xlo + ix * (E.cw - 1), xb = min(xa + E.cw - 1, E.xhi);
          const int ncw = xb - xa + 1;
          const int nkp = ((yb - ya + 1) * ncw + 15) & ~15;
          __syncthreads();
          load_chunk<DCH>(P, T, S.kbuf, L.rs, static_cast<const __nv_bfloat16*>(P.k), P.k_ld, z, ya, yb, xa, xb, nkp);
          __syncthreads();
          dense_scores<DCH, kWPG>(S.kbuf, L.rs, S.sbuf + static_cast<size_t>(r) * 16 * L.sld, L.sld, part, nkp, qa, qt);
          __syncthreads();
          if (!qvalid || zrel < zl_lo || zrel > zl_hi) continue;
          for (int j0 = js; j0 < je; j0 += 4) {
            unsigned long long vv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) vv[u] = (j0 + u < je) ? rec[j0 + u] : 0ull;
            bool hit[4];
            bool anyhit = false;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              hit[u] = (vv[u] >> 63) && static_cast<unsigned>(zrel - static_cast<int>((vv[u] >> 36) & 0x1fu)) <= 1u;
              anyhit |= hit[u];
            }
            if (!anyhit) continue;
            float acc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const Rec c = unpack_rec(vv[u], E);
              if (split && hit[u])
                hit[u] = axis_chunk_of(c.h0, E.ylo, E.R, E.ny) == iy && axis_chunk_of(c.w0, E.xlo, E.cw, E.nx) == ix;
              const float az = hit[u] ? frac_weight(c.ft, z != c.t0) : 0.f;
              const float ay0 = c.h0 < P.H ? 1.f - c.fh : 0.f, ay1 = c.h0 + 1 < P.H ? c.fh : 0.f;
              const float ax0 = c.w0 < P.W ? 1.f - c.fw : 0.f, ax1 = c.w0 + 1 < P.W ? c.fw : 0.f;
              // clamp the corner indices into the chunk so masked-out corners read a valid address
              const int k00 = hit[u] ? (c.h0 - ya) * ncw + (c.w0 - xa) : 0;
              const int k01 = (hit[u] && ax1 != 0.f) ? k00 + 1 : k00;
              const int k10 = (hit[u] && ay1 != 0.f) ? k00 + ncw : k00;
              const int k11 = (hit[u] && ax1 != 0.f && ay1 != 0.f) ? k00 + ncw + 1 : k00;
              float a = (ax0 * ay0) * az * srow_q[k00];
              a = fmaf((ax1 * ay0) * az, srow_q[k01], a);
              a = fmaf((ax0 * ay1) * az, srow_q[k10], a);
              acc[u] = fmaf((ax1 * ay1) * az, srow_q[k11], a);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (hit[u]) sacc[j0 + u] += acc[u];
          }
        }
      }
    }
  }

  // ---- extra keys: S_extra = Q . EK^T (all G keys in one chunk of the key buffer)
  if (P.G > 0) {
    const int gp = (P.G + 15) & ~15;
    __syncthreads();
    {
      const __nv_bfloat16* eb = static_cast<const __nv_bfloat16*>(P.ek) + static_cast<long long>(T.b) * P.G * P.e_ld + T.head * P.d;
      for (int idx = threadIdx.x; idx < gp * DCH; idx += kThreads) {
        const int key = idx / DCH, ch = idx - (idx / DCH) * DCH;
        __nv_bfloat16* dst = S.kbuf + static_cast<size_t>(key) * L.rs + ch * 8;
        if (key < P.G)
          cp_async16(smem_u32(dst), eb + static_cast<long long>(key) * P.e_ld + ch * 8);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
      cp_async_wait_all();
    }
    __syncthreads();
    dense_scores<DCH, kWPG>(S.kbuf, L.rs, S.sbuf + static_cast<size_t>(r) * 16 * L.sld, L.sld, part, gp, qa, qt);
    __syncthreads();
    for (int e = sub; e < P.G; e += kLPQ) sacc[K + e] = srow_q[e];
  }

  // ---- softmax over the K (+G) scores of each query (4 lanes per query)
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
  if (qvalid) {
    // optional per-sample softmax weights (normalised, before dropout) for the tensor-core backward
    float* prob_row = P.probs ? P.probs + ((static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow) * K : nullptr;
    const float inv_l = 1.f / l;
    for (int j = sub; j < KG; j += kLPQ) {
      const float p = exp2f(sacc[j] * P.scale_log2 - m);
      if (prob_row && j < K) prob_row[j] = p * inv_l;
      float pv = p;
      if (P.drop_thresh) {
        const uint64_t q = ((static_cast<uint64_t>(T.b) * P.T + T.tg) * P.H + qh) * P.W + qw;
        const uint64_t idx = (q * P.nh + T.head) * static_cast<uint64_t>(KG) + j;
        pv = dropout_keep(P.seed, idx, P.drop_thresh) ? p * P.drop_keep_scale : 0.f;
      }
      sacc[j] = pv;  // unnormalised, dropout applied
    }
  }
  if (sub == 0) {
    S.mrow[r * 16 + cq] = m;
    S.lrow[r * 16 + cq] = l;
    if (qvalid) P.lse[(static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow] = m + log2f(l);
  }

  // ---- pass 2: O = P~ . V
  constexpr int NT = DCH;  // n8 tiles of the head dimension, split over the group's warps
  constexpr int kTPW = (NT + kWPG - 1) / kWPG;
  const int nt0 = min(NT, part * kTPW), nt1 = min(NT, nt0 + kTPW);
  float o[kTPW + 1][4];  // o[j] accumulates d tile nt0 + j
#pragma unroll
  for (int i = 0; i < kTPW + 1; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float* prow = S.sbuf + static_cast<size_t>(r) * 16 * L.sld;
  float* prow_q = S.sbuf + (static_cast<size_t>(r) * 16 + cq) * L.sld;
  if (any && !chunk_overflow) {
    for (int z = E.zlo; z <= E.zhi; ++z) {
      const int zrel = z - E.zlo + 1;
      for (int iy = 0; iy < E.ny; ++iy) {
        const int ya = E.ylo + iy * (E.R - 1), yb = min(ya + E.R - 1, E.yhi);
        for (int ix = 0; ix < E.nx; ++ix) {
          const int xa = E.xlo + ix * (E.cw - 1), xb = min(xa + E.cw - 1, E.xhi);
          const int ncw = xb - xa + 1;
          const int nkp = ((yb - ya + 1) * ncw + 15) & ~15;
          __syncthreads();
          load_chunk<DCH>(P, T, S.kbuf, L.rs, static_cast<const __nv_bfloat16*>(P.v), P.v_ld, z, ya, yb, xa, xb, nkp);
          // zero P~ of the row group (16 rows x nkp), the group's warps split the rows
          for (int rrow = part * (16 / kWPG); rrow < (part + 1) * (16 / kWPG); ++rrow)
            for (int col = lane * 4; col < nkp; col += 128)
              *reinterpret_cast<float4*>(prow + static_cast<size_t>(rrow) * L.sld + col) = make_float4(0.f, 0.f, 0.f, 0.f);
          __syncthreads();
          if (qvalid && zrel >= zl_lo && zrel <= zl_hi) {
            unsigned int* prow_u = reinterpret_cast<unsigned int*>(prow_q);
            for (int j0 = js; j0 < je; j0 += 4) {
              unsigned long long vv[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) vv[u] = (j0 + u < je) ? rec[j0 + u] : 0ull;
              bool hit[4];
              bool anyhit = false;
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                hit[u] = (vv[u] >> 63) && static_cast<unsigned>(zrel - static_cast<int>((vv[u] >> 36) & 0x1fu)) <= 1u;
                anyhit |= hit[u];
              }
              if (!anyhit) continue;
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                if (!hit[u]) continue;
                const Rec c = unpack_rec(vv[u], E);
                if (split && (axis_chunk_of(c.h0, E.ylo, E.R, E.ny) != iy || axis_chunk_of(c.w0, E.xlo, E.cw, E.nx) != ix))
                  continue;
                const float pv = sacc[j0 + u] * kPtScale;
                if (pv == 0.f) continue;
                const float az = frac_weight(c.ft, z != c.t0);
                const int k00 = (c.h0 - ya) * ncw + (c.w0 - xa);
                const float ay0 = 1.f - c.fh, ay1 = c.fh, ax0 = 1.f - c.fw, ax1 = c.fw;
                atomicAdd(prow_u + k00, __float2uint_rn(pv * ((ax0 * ay0) * az)));
                if (c.w0 + 1 < P.W) atomicAdd(prow_u + k00 + 1, __float2uint_rn(pv * ((ax1 * ay0) * az)));
                if (c.h0 + 1 < P.H) {
                  atomicAdd(prow_u + k00 + ncw, __float2uint_rn(pv * ((ax0 * ay1) * az)));
                  if (c.w0 + 1 < P.W) atomicAdd(prow_u + k00 + ncw + 1, __float2uint_rn(pv * ((ax1 * ay1) * az)));
                }
              }
            }
          }
          __syncthreads();
          av_product<DCH, kTPW, true>(prow, L.sld, S.kbuf, L.rs, nt0, nt1, nkp, o);
        }
      }
    }
  }
  if (P.G > 0) {
    const int gp = (P.G + 15) & ~15;
    __syncthreads();
    {
      const __nv_bfloat16* eb = static_cast<const __nv_bfloat16*>(P.ev) + static_cast<long long>(T.b) * P.G * P.e_ld + T.head * P.d;
      for (int idx = threadIdx.x; idx < gp * DCH; idx += kThreads) {
        const int key = idx / DCH, ch = idx - (idx / DCH) * DCH;
        __nv_bfloat16* dst = S.kbuf + static_cast<size_t>(key) * L.rs + ch * 8;
        if (key < P.G)
          cp_async16(smem_u32(dst), eb + static_cast<long long>(key) * P.e_ld + ch * 8);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
      cp_async_wait_all();
    }
    for (int rrow = part * (16 / kWPG); rrow < (part + 1) * (16 / kWPG); ++rrow)
      for (int col = lane * 4; col < gp; col += 128)
        *reinterpret_cast<float4*>(prow + static_cast<size_t>(rrow) * L.sld + col) = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    for (int e = sub; e < P.G; e += kLPQ)
      reinterpret_cast<unsigned int*>(prow_q)[e] = qvalid ? __float2uint_rn(sacc[K + e] * kPtScale) : 0u;
    __syncthreads();
    av_product<DCH, kTPW, true>(prow, L.sld, S.kbuf, L.rs, nt0, nt1, gp, o);
  }

  // ---- normalise and store
  __syncthreads();  // lrow written by the sample lanes of other warps
  {
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

}  // namespace tc

// ------------------------------------------------------------------------------ host side
bool tc_supported(const AttnParams& P) {
  if (P.dtype != MSL_DTYPE_BF16) return false;
  if (P.d % 8 != 0 || P.d < 16 || P.d > 128) return false;
  if (P.T > 65535 || P.K > 2048 || P.G > 256) return false;
  if (P.drop_thresh && P.drop_keep_scale > 10.f) return false;  // fixed-point P~ range (dropout p <= 0.9)
  // base-grid tables hold at most 96 positions per axis
  if (P.kt > 96 || P.kh + tc::kTileH - 1 > 96 || P.kw + tc::kTileW - 1 > 96) return false;
  return true;
}

bool tc_plan(const AttnParams& P, TcLaunch& L, int smem_limit) {
  const int dch = P.d / 8;
  L.rs = (dch & 1) ? P.d : P.d + 8;  // odd number of 16-byte chunks per row: conflict-free ldmatrix
  L.tiles_h = (P.H + tc::kTileH - 1) / tc::kTileH;
  L.tiles_w = (P.W + tc::kTileW - 1) / tc::kTileW;
  const size_t fixed = static_cast<size_t>(tc::kQ) * (P.K + P.G) * 4 + static_cast<size_t>(tc::kQ) * P.K * 8 +
                       tc::kEnvWords * 4 + 2 * tc::kQ * 4 + 256;
  const size_t per_key = static_cast<size_t>(L.rs) * 2 + 4 * 16 * 4;
  if (fixed + per_key * 64 > static_cast<size_t>(smem_limit)) return false;
  int mk = static_cast<int>((static_cast<size_t>(smem_limit) - fixed - 4 * 16 * 8 * 4) / per_key);
  mk &= ~15;
  const int gp = (P.G + 15) & ~15;
  if (mk < 64 || mk < gp) return false;
  if (mk > 1024) mk = 1024;
  L.maxkeys = mk;
  L.sld = mk + 8;
  // the setup stages 32 queries x K x 3 offsets in the key + score buffers
  if (static_cast<size_t>(mk) * L.rs * 2 + static_cast<size_t>(4) * 16 * L.sld * 4 < static_cast<size_t>(32) * P.K * 12)
    return false;  // row stride = 8 or 24 (mod 32) words: mma fragment rows hit distinct banks
  L.smem = static_cast<size_t>(mk) * L.rs * 2 + static_cast<size_t>(4) * 16 * L.sld * 4 + fixed;
  L.tiles = static_cast<long long>(P.B) * P.q_frames * L.tiles_h * L.tiles_w * P.nh;
  return L.tiles <= 0x7fffffffLL;
}

template <int DCH>
static cudaError_t launch_fwd_tc_t(const AttnParams& P, const TcLaunch& L, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(tc::dsa_fwd_tc_kernel<DCH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  tc::dsa_fwd_tc_kernel<DCH><<<static_cast<unsigned>(L.tiles), tc::kThreads, L.smem, s>>>(P, L);
  return cudaGetLastError();
}

cudaError_t launch_attn_fwd_tc(const AttnParams& P, const TcLaunch& L, cudaStream_t s) {
  switch (P.d / 8) {
    case 2: return launch_fwd_tc_t<2>(P, L, s);
    case 3: return launch_fwd_tc_t<3>(P, L, s);
    case 4: return launch_fwd_tc_t<4>(P, L, s);
    case 5: return launch_fwd_tc_t<5>(P, L, s);
    case 6: return launch_fwd_tc_t<6>(P, L, s);
    case 7: return launch_fwd_tc_t<7>(P, L, s);
    case 8: return launch_fwd_tc_t<8>(P, L, s);
    case 9: return launch_fwd_tc_t<9>(P, L, s);
    case 10: return launch_fwd_tc_t<10>(P, L, s);
    case 11: return launch_fwd_tc_t<11>(P, L, s);
    case 12: return launch_fwd_tc_t<12>(P, L, s);
    case 13: return launch_fwd_tc_t<13>(P, L, s);
    case 14: return launch_fwd_tc_t<14>(P, L, s);
    case 15: return launch_fwd_tc_t<15>(P, L, s);
    case 16: return launch_fwd_tc_t<16>(P, L, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace msl
