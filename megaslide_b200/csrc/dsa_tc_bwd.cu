// Tensor-core ("key envelope") backward of the deformable gather attention, bf16, no extra keys.
//
// One CTA owns a tile of 4 x 8 queries of one frame, one head and one sample (32 queries = two
// 16-query row groups; 16 warps, 8 per group; 16 lanes per query for the per-sample work).  Besides
// the forward's inputs it reads dO (gradient of the attention output), the forward output O and the
// forward's per-sample softmax weights p (`probs`).  With D = dO . O per query and, per window sample
// j with trilinear corners c and weights w_c, pv_j = p_j * keep_j / (1 - p_drop):
//
//   pass 1, per envelope chunk (V side):  dP = dO . V_chunk^T on the tensor cores; every sample adds
//            dp_j  += sum_c w_c dP[q, c]                     (dp_j = dO . v_j, before dropout)
//            g_j   += pv_j * sum_c (dw_c / dpix) dP[q, c]    (coordinate gradient, value part)
//   then     dsq_j = softmax_scale * p_j * (keep_j dp_j / (1 - p_drop) - D)
//   pass 2, per envelope chunk (K side):  S = Q . K_chunk^T; every sample adds
//            g_j   += dsq_j * sum_c (dw_c / dpix) S[q, c]    (coordinate gradient, key part)
//            scatter dsq_j w_c into dS~[q, key]:  dQ += dS~ . K_chunk,  dK_chunk = dS~^T . Q
//            scatter pv_j  w_c into P~[q, key]:   dV_chunk = P~^T . dO
//   dK / dV chunks are added to the float32 accumulators with vector atomics (one per 4 channels of
//   a key that received anything); g_j becomes the offset gradient through grid_sample's clip rule
//   and the offset normalisation, with the reference's axis swap.
//
// Reference semantics: autograd of infinity/video/attention.py:113-186 (grid_sampler_3d_backward,
// bmm and softmax backward, dropout).

#include "dsa_tc.cuh"

namespace msl {
namespace tc {
namespace bwd {

constexpr int kGroups = 2;                  // 16-query row groups per tile
constexpr int kWPG = kWarps / kGroups;      // warps per row group
constexpr int kLPQ = kWPG * 32 / 16;        // lanes per query
constexpr int kTileH = 4, kQ = kTileH * kTileW;

// record flags: grid coordinate strictly inside (0, S-1) along t / h / w, dropout keep
constexpr int kBitInT = 57, kBitInH = 58, kBitInW = 59, kBitKeep = 60;

struct Smem {
  __nv_bfloat16* kbuf;      // [maxkeys][rs]   K or V chunk (setup: staged offsets, spilling into sbuf)
  float* sbuf;              // [32][sld]       dP / S, then dS~, then P~ (u32 fixed point)
  __nv_bfloat16* qs;        // [32][rs]        Q rows of the tile
  __nv_bfloat16* dos;       // [32][rs]        dO rows of the tile
  unsigned long long* rec;  // [32][K]         packed sample records
  float* pp;                // [32][K]         p_j
  float* acc;               // [32][K]         dp_j, then dsq_j
  float* g3;                // [32][K][3]      coordinate gradient (t, h, w) before the clip rule
  int* env;                 // envelope + base-grid tables
  float* dd;                // [32]            D = dO . O
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
  s.dos = reinterpret_cast<__nv_bfloat16*>(base + off);
  off += static_cast<size_t>(kQ) * L.rs * 2;
  s.rec = reinterpret_cast<unsigned long long*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 8;
  s.pp = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 4;
  s.acc = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 4;
  s.g3 = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 12;
  s.env = reinterpret_cast<int*>(base + off);
  off += kEnvWords * 4;
  s.dd = reinterpret_cast<float*>(base + off);
  return s;
}

// shared memory besides the key buffer and the score rows
size_t smem_fixed(const AttnParams& P, int rs) {
  return static_cast<size_t>(kQ) * rs * 2 * 2 + static_cast<size_t>(kQ) * P.K * (8 + 4 + 4 + 12) + kEnvWords * 4 +
         kQ * 4 + 256;
}

// In-plane terms of one sample in one frame from a row of per-key values (corners outside the
// volume count as 0, like grid_sample's zero contribution of out-of-bounds corners):
//   bil = sum_c wy_c wx_c v_c,  dvx = d bil / d pw,  dvy = d bil / d ph.
struct PlaneTerms {
  float bil, dvx, dvy;
};

__device__ __forceinline__ PlaneTerms plane_terms(const float* row, int k00, int ncw, const Rec& c, int H, int W) {
  const bool xok = c.w0 + 1 < W, yok = c.h0 + 1 < H;
  const float v00 = row[k00];
  const float v01 = xok ? row[k00 + 1] : 0.f;
  const float v10 = yok ? row[k00 + ncw] : 0.f;
  const float v11 = (xok && yok) ? row[k00 + ncw + 1] : 0.f;
  const float ax0 = 1.f - c.fw, ax1 = c.fw, ay0 = 1.f - c.fh, ay1 = c.fh;
  PlaneTerms t;
  t.bil = ay0 * (ax0 * v00 + ax1 * v01) + ay1 * (ax0 * v10 + ax1 * v11);
  t.dvx = ay0 * (v01 - v00) + ay1 * (v11 - v10);
  t.dvy = ax0 * (v10 - v00) + ax1 * (v11 - v01);
  return t;
}

// accum[key][d] += A^T . X for one envelope chunk: A = the tile's 32 dense rows in sbuf (fp32, or u32
// fixed point when FIXED), X = 32 bf16 rows (Q or dO) in shared memory.  Items (16-key tile, group of
// 8-channel tiles) are spread over the 16 warps; each result row is added to the float32 accumulator
// of its key with one float4 atomic per 4 channels, skipped when all four are zero.
template <int DCH, bool FIXED>
__device__ __forceinline__ void kv_product_flush(const AttnParams& P, const TileCtx& T, const TcLaunch& L,
                                                 const float* sbuf, const __nv_bfloat16* xs, int nkp, int nk, int ncw,
                                                 int ya, int xa, int zl, float* accum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  constexpr int NP = (DCH + 1) / 2;  // 16-channel pairs of 8-channel tiles
  const int mtiles = nkp >> 4;
  int ns = (kWarps + mtiles - 1) / mtiles;  // channel splits per key tile
  if (ns > NP) ns = NP;
  const int ppi = (NP + ns - 1) / ns;  // pairs per item
  const int items = mtiles * ns;
  for (int item = warp; item < items; item += kWarps) {
    const int mt = item / ns, sp = item - (item / ns) * ns;
    const int p0 = sp * ppi, p1 = min(NP, p0 + ppi);
    // A fragments: rows = keys mt*16 + (g, g+8), columns = queries (two k16 steps)
    uint32_t a[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const float* c0 = sbuf + static_cast<size_t>(kk * 16 + 2 * t4) * L.sld + mt * 16 + g;
      const float* c1 = c0 + L.sld;
      const float* c8 = c0 + static_cast<size_t>(8) * L.sld;
      const float* c9 = c8 + L.sld;
      float v[8] = {c0[0], c1[0], c0[8], c1[8], c8[0], c9[0], c8[8], c9[8]};
      if constexpr (FIXED) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = static_cast<float>(__float_as_uint(v[i])) * kPtInv;
      }
      a[kk][0] = pack_bf16(v[0], v[1]);  // (key g,   queries 2t4, 2t4+1)
      a[kk][1] = pack_bf16(v[2], v[3]);  // (key g+8, queries 2t4, 2t4+1)
      a[kk][2] = pack_bf16(v[4], v[5]);  // (key g,   queries 2t4+8, +9)
      a[kk][3] = pack_bf16(v[6], v[7]);  // (key g+8, queries 2t4+8, +9)
    }
    // destination rows of keys mt*16 + g and mt*16 + g + 8 (padding keys are skipped)
    const int k0 = mt * 16 + g, k1 = k0 + 8;
    float* dst0 = nullptr;
    float* dst1 = nullptr;
    if (k0 < nk) {
      const int y = ya + k0 / ncw, x = xa + k0 % ncw;
      dst0 = accum + (static_cast<long long>(T.b) * P.Nkv + (static_cast<long long>(zl) * P.H + y) * P.W + x) * P.acc_ld +
             T.head * P.d;
    }
    if (k1 < nk) {
      const int y = ya + k1 / ncw, x = xa + k1 % ncw;
      dst1 = accum + (static_cast<long long>(T.b) * P.Nkv + (static_cast<long long>(zl) * P.H + y) * P.W + x) * P.acc_ld +
             T.head * P.d;
    }
    for (int pr = p0; pr < p1; ++pr) {
      const int nt = 2 * pr;
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const bool two = nt + 1 < DCH;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        // x4.trans matrices: (queries +0..7, ch nt) (queries +8..15, ch nt) (queries +0..7, ch nt+1) (+8..15, nt+1)
        const __nv_bfloat16* rowp = xs + static_cast<size_t>(kk * 16 + rr + ((mi & 1) ? 8 : 0)) * L.rs;
        if (two) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(rowp + (nt + (mi >> 1)) * 8), b0, b1, b2, b3);
          mma16816(c[0], a[kk], b0, b1);
          mma16816(c[1], a[kk], b2, b3);
        } else {
          uint32_t b0, b1;
          ldsm_x2_t(smem_u32(rowp + nt * 8), b0, b1);
          mma16816(c[0], a[kk], b0, b1);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 1 && !two) break;
        // lanes t4 = 0, 2 flush key g (channels 2t4..2t4+3), lanes t4 = 1, 3 key g + 8 (2t4-2..2t4+1)
        const float o0 = __shfl_xor_sync(kFull, c[h][0], 1), o1 = __shfl_xor_sync(kFull, c[h][1], 1);
        const float o2 = __shfl_xor_sync(kFull, c[h][2], 1), o3 = __shfl_xor_sync(kFull, c[h][3], 1);
        const int ch = (nt + h) * 8;
        if ((t4 & 1) == 0) {
          const float4 v = make_float4(c[h][0], c[h][1], o0, o1);
          if (dst0 && (v.x != 0.f || v.y != 0.f || v.z != 0.f || v.w != 0.f))
            atomicAdd(reinterpret_cast<float4*>(dst0 + ch + 2 * t4), v);
        } else {
          const float4 v = make_float4(o2, o3, c[h][2], c[h][3]);
          if (dst1 && (v.x != 0.f || v.y != 0.f || v.z != 0.f || v.w != 0.f))
            atomicAdd(reinterpret_cast<float4*>(dst1 + ch + 2 * t4 - 2), v);
        }
      }
    }
  }
}

template <int DCH>
__global__ void __launch_bounds__(kThreads, 1) dsa_bwd_tc_kernel(const AttnParams P, const TcLaunch L) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const Smem S = carve(smem_raw, P, L);
  const TileCtx T = decode_tile(P, L, kTileH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp / kWPG, part = warp - (warp / kWPG) * kWPG;
  const int ll = part * 32 + lane;
  const int cq = ll / kLPQ, sub = ll - (ll / kLPQ) * kLPQ;
  const int K = P.K;
  // the lanes of a query own contiguous window ranges (few frames per lane)
  const int jper = (K + kLPQ - 1) / kLPQ;
  const int js = min(K, sub * jper), je = min(K, js + jper);
  const int qi = r * 16 + cq;  // owned query within the tile

  int qh, qw;
  query_hw(T, r, cq, qh, qw);
  const bool qvalid = qh < P.H && qw < P.W;
  const long long qrow = (static_cast<long long>(T.tl) * P.H + qh) * P.W + qw;
  unsigned long long* rec = S.rec + static_cast<size_t>(qi) * K;
  float* pp = S.pp + static_cast<size_t>(qi) * K;
  float* acc = S.acc + static_cast<size_t>(qi) * K;
  float* g3 = S.g3 + static_cast<size_t>(qi) * K * 3;

  float* tabz = reinterpret_cast<float*>(S.env + 16);
  float* taby = tabz + 96;
  float* tabx = taby + 96;
  if (threadIdx.x == 0) {
    S.env[0] = 0x7fffffff; S.env[1] = -0x7fffffff; S.env[2] = 0x7fffffff;
    S.env[3] = -0x7fffffff; S.env[4] = 0x7fffffff; S.env[5] = -0x7fffffff;
  }
  fill_tabs(P, T, kTileH, tabz, taby, tabx);

  // ---- stage the tile's offsets (this head), Q and dO rows with one wave of cp.async
  const int K3 = 3 * K;
  float* ostage = reinterpret_cast<float*>(S.kbuf);
  for (int q2 = warp; q2 < kQ; q2 += kWarps) {
    int sqh, sqw;
    query_hw(T, q2 >> 4, q2 & 15, sqh, sqw);
    const bool ok = sqh < P.H && sqw < P.W;
    const long long grow = static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + sqh) * P.W + sqw;
    if (ok) {
      const float* src = P.offsets + grow * P.off_ld + static_cast<long long>(T.head) * K3;
      float* dst = ostage + static_cast<size_t>(q2) * K3;
      for (int k = lane; k < K3; k += 32) cp_async4(smem_u32(dst + k), src + k);
    }
    for (int ch = lane; ch < DCH; ch += 32) {
      __nv_bfloat16* dq_ = S.qs + static_cast<size_t>(q2) * L.rs + ch * 8;
      __nv_bfloat16* dd_ = S.dos + static_cast<size_t>(q2) * L.rs + ch * 8;
      if (ok) {
        cp_async16(smem_u32(dq_), static_cast<const __nv_bfloat16*>(P.q) + grow * P.q_ld + T.head * P.d + ch * 8);
        cp_async16(smem_u32(dd_), static_cast<const __nv_bfloat16*>(P.dout) + grow * P.dout_ld + T.head * P.d + ch * 8);
      } else {
        *reinterpret_cast<uint4*>(dq_) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(dd_) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
  cp_async_wait_all();
  __syncthreads();
  const Tabs tb{tabz, taby, tabx};
  const int qy = qh - T.qh0, qx = qw - T.qw0;

  // ---- D = dO . O per query (the lanes of a query split the head dimension)
  {
    float dpart = 0.f;
    if (qvalid) {
      const __nv_bfloat16* orow_g = static_cast<const __nv_bfloat16*>(P.out) +
                                    (static_cast<long long>(T.b) * P.Nq + qrow) * P.out_ld + T.head * P.d;
      const __nv_bfloat16* drow_s = S.dos + static_cast<size_t>(qi) * L.rs;
      for (int i = sub; i < P.d; i += kLPQ)
        dpart = fmaf(__bfloat162float(orow_g[i]), __bfloat162float(drow_s[i]), dpart);
    }
#pragma unroll
    for (int o = 1; o < kLPQ; o <<= 1) dpart += __shfl_xor_sync(kFull, dpart, o);
    if (sub == 0) S.dd[qi] = dpart;
  }

  // ---- sample coordinates -> envelope (raw coordinates parked in rec / acc)
  const int kvlo = max(P.kv_frame0, 0), kvhi = min(P.kv_frame0 + P.kv_frames, P.T) - 1;
  int zmn = 0x7fffffff, zmx = -0x7fffffff, ymn = 0x7fffffff, ymx = -0x7fffffff, xmn = 0x7fffffff, xmx = -0x7fffffff;
  bool miss = false;
  if (qvalid) {
    const float* oq = ostage + static_cast<size_t>(qi) * K3;
    WinIdx wi;
    wi.init(js, P.kh, P.kw);
    for (int j = js; j < je; ++j, wi.advance(1, P.kh, P.kw)) {
      float pt, ph, pw;
      tab_coords(P, tb, qy, qx, wi.it, wi.ih, wi.iw, oq[3 * j], oq[3 * j + 1], oq[3 * j + 2], pt, ph, pw);
      rec[j] = (static_cast<unsigned long long>(__float_as_uint(ph)) << 32) | __float_as_uint(pt);
      acc[j] = pw;
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
  const bool overflow = any && (E.zhi - E.zlo + 2 > 31 || E.yhi - E.ylo > 255 || E.xhi - E.xlo > 255);
  if (overflow && threadIdx.x == 0 && P.status) atomicOr(P.status, MSL_STATUS_TC_RANGE);

  // ---- records (with interior and keep flags), p_j, cleared accumulators
  int zl_lo = 0x7fff, zl_hi = -1;
  if (qvalid) {
    const float* prob_row = P.probs + ((static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow) * K;
    const uint64_t qglob = ((static_cast<uint64_t>(T.b) * P.T + T.tg) * P.H + qh) * P.W + qw;
    for (int j = js; j < je; ++j) {
      const unsigned long long raw = rec[j];
      const float pt = __uint_as_float(static_cast<uint32_t>(raw)), ph = __uint_as_float(static_cast<uint32_t>(raw >> 32));
      const float pw = acc[j];
      acc[j] = 0.f;
      g3[3 * j] = 0.f;
      g3[3 * j + 1] = 0.f;
      g3[3 * j + 2] = 0.f;
      pp[j] = __ldg(prob_row + j);
      const int t0 = static_cast<int>(floorf(pt)), h0 = static_cast<int>(floorf(ph)), w0 = static_cast<int>(floorf(pw));
      if (!any || overflow || t0 + 1 < E.zlo || t0 > E.zhi) {  // no corner in a frame the K/V buffers hold
        rec[j] = 0ull;
        continue;
      }
      bool keep = true;
      if (P.drop_thresh)
        keep = dropout_keep(P.seed, (qglob * P.nh + T.head) * static_cast<uint64_t>(K + P.G) + j, P.drop_thresh);
      const unsigned long long flags = (clip_grad_mult(pt, P.T) != 0.f ? 1ull << kBitInT : 0ull) |
                                       (clip_grad_mult(ph, P.H) != 0.f ? 1ull << kBitInH : 0ull) |
                                       (clip_grad_mult(pw, P.W) != 0.f ? 1ull << kBitInW : 0ull) |
                                       (keep ? 1ull << kBitKeep : 0ull);
      rec[j] = pack_rec(pt - static_cast<float>(t0), ph - static_cast<float>(h0), pw - static_cast<float>(w0),
                        t0 - E.zlo + 1, h0 - E.ylo, w0 - E.xlo) |
               flags;
      zl_lo = min(zl_lo, t0 - E.zlo + 1);
      zl_hi = max(zl_hi, t0 - E.zlo + 2);
    }
  }

  // ---- A fragments of dO and Q (rows g and g + 8 of the row group) from the staged rows
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t da[DCH / 2 > 0 ? DCH / 2 : 1][4], dt_[2] = {0u, 0u};
  uint32_t qa[DCH / 2 > 0 ? DCH / 2 : 1][4], qt[2] = {0u, 0u};
  {
    const __nv_bfloat16* d0 = S.dos + static_cast<size_t>(r * 16 + g) * L.rs;
    const __nv_bfloat16* d1 = S.dos + static_cast<size_t>(r * 16 + g + 8) * L.rs;
    const __nv_bfloat16* q0 = S.qs + static_cast<size_t>(r * 16 + g) * L.rs;
    const __nv_bfloat16* q1 = S.qs + static_cast<size_t>(r * 16 + g + 8) * L.rs;
#pragma unroll
    for (int ks = 0; ks < DCH / 2; ++ks) {
      da[ks][0] = *reinterpret_cast<const uint32_t*>(d0 + ks * 16 + 2 * t4);
      da[ks][1] = *reinterpret_cast<const uint32_t*>(d1 + ks * 16 + 2 * t4);
      da[ks][2] = *reinterpret_cast<const uint32_t*>(d0 + ks * 16 + 8 + 2 * t4);
      da[ks][3] = *reinterpret_cast<const uint32_t*>(d1 + ks * 16 + 8 + 2 * t4);
      qa[ks][0] = *reinterpret_cast<const uint32_t*>(q0 + ks * 16 + 2 * t4);
      qa[ks][1] = *reinterpret_cast<const uint32_t*>(q1 + ks * 16 + 2 * t4);
      qa[ks][2] = *reinterpret_cast<const uint32_t*>(q0 + ks * 16 + 8 + 2 * t4);
      qa[ks][3] = *reinterpret_cast<const uint32_t*>(q1 + ks * 16 + 8 + 2 * t4);
    }
    if constexpr (DCH & 1) {
      dt_[0] = *reinterpret_cast<const uint32_t*>(d0 + (DCH - 1) * 8 + 2 * t4);
      dt_[1] = *reinterpret_cast<const uint32_t*>(d1 + (DCH - 1) * 8 + 2 * t4);
      qt[0] = *reinterpret_cast<const uint32_t*>(q0 + (DCH - 1) * 8 + 2 * t4);
      qt[1] = *reinterpret_cast<const uint32_t*>(q1 + (DCH - 1) * 8 + 2 * t4);
    }
  }
  float* grow_s = S.sbuf + static_cast<size_t>(r) * 16 * L.sld;  // the row group's 16 dense rows
  float* srow_q = S.sbuf + static_cast<size_t>(qi) * L.sld;     // the owned query's dense row

  // ---- pass 1: V side (dp_j and the value part of the coordinate gradient)
  if (any && !overflow) {
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
          __syncthreads();
          dense_scores<DCH, kWPG>(S.kbuf, L.rs, grow_s, L.sld, part, nkp, da, dt_);
          __syncthreads();
          if (!qvalid || zrel < zl_lo || zrel > zl_hi) continue;
          for (int j = js; j < je; ++j) {
            const unsigned long long v = rec[j];
            if (!rec_in_plane(v, zrel)) continue;
            const Rec c = unpack_rec(v, E);
            if (split && (axis_chunk_of(c.h0, E.ylo, E.R, E.ny) != iy || axis_chunk_of(c.w0, E.xlo, E.cw, E.nx) != ix))
              continue;
            const bool upper = z != c.t0;
            const float az = frac_weight(c.ft, upper);
            const PlaneTerms pt_ = plane_terms(srow_q, (c.h0 - ya) * ncw + (c.w0 - xa), ncw, c, P.H, P.W);
            const float pv = ((v >> kBitKeep) & 1ull) ? pp[j] * P.drop_keep_scale : 0.f;
            acc[j] = fmaf(az, pt_.bil, acc[j]);
            g3[3 * j + 0] = fmaf(pv, upper ? pt_.bil : -pt_.bil, g3[3 * j + 0]);
            g3[3 * j + 1] = fmaf(pv * az, pt_.dvy, g3[3 * j + 1]);
            g3[3 * j + 2] = fmaf(pv * az, pt_.dvx, g3[3 * j + 2]);
          }
        }
      }
    }
  }

  // ---- dsq_j = softmax_scale * p_j * (keep_j dp_j / (1 - p_drop) - D)
  if (qvalid) {
    const float D = S.dd[qi];
    for (int j = js; j < je; ++j) {
      const float kf = ((rec[j] >> kBitKeep) & 1ull) ? P.drop_keep_scale : 0.f;
      acc[j] = pp[j] * fmaf(kf, acc[j], -D) * P.scale;
    }
  }

  // ---- pass 2: K side (key part of the coordinate gradient, dQ, dK, dV)
  constexpr int kTPW = (DCH + kWPG - 1) / kWPG;  // dQ channel tiles per warp
  const int nt0 = min(DCH, part * kTPW), nt1 = min(DCH, nt0 + kTPW);
  float oq[kTPW + 1][4];
#pragma unroll
  for (int i = 0; i < kTPW + 1; ++i) oq[i][0] = oq[i][1] = oq[i][2] = oq[i][3] = 0.f;
  if (any && !overflow) {
    for (int z = E.zlo; z <= E.zhi; ++z) {
      const int zrel = z - E.zlo + 1;
      const int zl = z - P.kv_frame0;
      const bool lane_active = qvalid && zrel >= zl_lo && zrel <= zl_hi;
      for (int iy = 0; iy < E.ny; ++iy) {
        const int ya = E.ylo + iy * (E.R - 1), yb = min(ya + E.R - 1, E.yhi);
        for (int ix = 0; ix < E.nx; ++ix) {
          const int xa = E.xlo + ix * (E.cw - 1), xb = min(xa + E.cw - 1, E.xhi);
          const int ncw = xb - xa + 1;
          const int nk = (yb - ya + 1) * ncw;
          const int nkp = (nk + 15) & ~15;
          __syncthreads();
          load_chunk<DCH>(P, T, S.kbuf, L.rs, static_cast<const __nv_bfloat16*>(P.k), P.k_ld, z, ya, yb, xa, xb, nkp);
          __syncthreads();
          dense_scores<DCH, kWPG>(S.kbuf, L.rs, grow_s, L.sld, part, nkp, qa, qt);
          __syncthreads();
          if (lane_active) {
            for (int j = js; j < je; ++j) {
              const unsigned long long v = rec[j];
              if (!rec_in_plane(v, zrel)) continue;
              const Rec c = unpack_rec(v, E);
              if (split && (axis_chunk_of(c.h0, E.ylo, E.R, E.ny) != iy || axis_chunk_of(c.w0, E.xlo, E.cw, E.nx) != ix))
                continue;
              const bool upper = z != c.t0;
              const float az = frac_weight(c.ft, upper);
              const PlaneTerms pt_ = plane_terms(srow_q, (c.h0 - ya) * ncw + (c.w0 - xa), ncw, c, P.H, P.W);
              const float dsq = acc[j];
              g3[3 * j + 0] = fmaf(dsq, upper ? pt_.bil : -pt_.bil, g3[3 * j + 0]);
              g3[3 * j + 1] = fmaf(dsq * az, pt_.dvy, g3[3 * j + 1]);
              g3[3 * j + 2] = fmaf(dsq * az, pt_.dvx, g3[3 * j + 2]);
            }
          }
          __syncthreads();
          // dS~ (float atomics: dsq is signed)
          for (int row = warp; row < kQ; row += kWarps)
            for (int col = lane * 4; col < nkp; col += 128)
              *reinterpret_cast<float4*>(S.sbuf + static_cast<size_t>(row) * L.sld + col) = make_float4(0.f, 0.f, 0.f, 0.f);
          __syncthreads();
          if (lane_active) {
            for (int j = js; j < je; ++j) {
              const unsigned long long v = rec[j];
              if (!rec_in_plane(v, zrel)) continue;
              const Rec c = unpack_rec(v, E);
              if (split && (axis_chunk_of(c.h0, E.ylo, E.R, E.ny) != iy || axis_chunk_of(c.w0, E.xlo, E.cw, E.nx) != ix))
                continue;
              const float dsq = acc[j] * frac_weight(c.ft, z != c.t0);
              const int k00 = (c.h0 - ya) * ncw + (c.w0 - xa);
              const float ax0 = 1.f - c.fw, ax1 = c.fw, ay0 = 1.f - c.fh, ay1 = c.fh;
              atomicAdd(srow_q + k00, dsq * (ax0 * ay0));
              if (c.w0 + 1 < P.W) atomicAdd(srow_q + k00 + 1, dsq * (ax1 * ay0));
              if (c.h0 + 1 < P.H) {
                atomicAdd(srow_q + k00 + ncw, dsq * (ax0 * ay1));
                if (c.w0 + 1 < P.W) atomicAdd(srow_q + k00 + ncw + 1, dsq * (ax1 * ay1));
              }
            }
          }
          __syncthreads();
          // dQ += dS~ . K_chunk (row group r, channel tiles [nt0, nt1)) and dK_chunk = dS~^T . Q
          av_product<DCH, kTPW, false>(grow_s, L.sld, S.kbuf, L.rs, nt0, nt1, nkp, oq);
          kv_product_flush<DCH, false>(P, T, L, S.sbuf, S.qs, nkp, nk, ncw, ya, xa, zl, P.dk_acc);
          __syncthreads();
          // P~ (fixed point, pv >= 0) -> dV_chunk = P~^T . dO
          for (int row = warp; row < kQ; row += kWarps)
            for (int col = lane * 4; col < nkp; col += 128)
              *reinterpret_cast<float4*>(S.sbuf + static_cast<size_t>(row) * L.sld + col) = make_float4(0.f, 0.f, 0.f, 0.f);
          __syncthreads();
          if (lane_active) {
            unsigned int* prow_u = reinterpret_cast<unsigned int*>(srow_q);
            for (int j = js; j < je; ++j) {
              const unsigned long long v = rec[j];
              if (!rec_in_plane(v, zrel) || !((v >> kBitKeep) & 1ull)) continue;
              const Rec c = unpack_rec(v, E);
              if (split && (axis_chunk_of(c.h0, E.ylo, E.R, E.ny) != iy || axis_chunk_of(c.w0, E.xlo, E.cw, E.nx) != ix))
                continue;
              const float pv = pp[j] * P.drop_keep_scale * frac_weight(c.ft, z != c.t0) * kPtScale;
              const int k00 = (c.h0 - ya) * ncw + (c.w0 - xa);
              const float ax0 = 1.f - c.fw, ax1 = c.fw, ay0 = 1.f - c.fh, ay1 = c.fh;
              atomicAdd(prow_u + k00, __float2uint_rn(pv * (ax0 * ay0)));
              if (c.w0 + 1 < P.W) atomicAdd(prow_u + k00 + 1, __float2uint_rn(pv * (ax1 * ay0)));
              if (c.h0 + 1 < P.H) {
                atomicAdd(prow_u + k00 + ncw, __float2uint_rn(pv * (ax0 * ay1)));
                if (c.w0 + 1 < P.W) atomicAdd(prow_u + k00 + ncw + 1, __float2uint_rn(pv * (ax1 * ay1)));
              }
            }
          }
          __syncthreads();
          kv_product_flush<DCH, true>(P, T, L, S.sbuf, S.dos, nkp, nk, ncw, ya, xa, zl, P.dv_acc);
        }
      }
    }
  }

  // ---- dQ (bf16) and the offset gradients
  {
    int qh0_, qw0_, qh1_, qw1_;
    query_hw(T, r, g, qh0_, qw0_);
    query_hw(T, r, g + 8, qh1_, qw1_);
    const bool v0 = qh0_ < P.H && qw0_ < P.W, v1 = qh1_ < P.H && qw1_ < P.W;
    __nv_bfloat16* o0 = static_cast<__nv_bfloat16*>(P.dq) +
        (static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + qh0_) * P.W + qw0_) * P.dq_ld + T.head * P.d;
    __nv_bfloat16* o1 = static_cast<__nv_bfloat16*>(P.dq) +
        (static_cast<long long>(T.b) * P.Nq + (static_cast<long long>(T.tl) * P.H + qh1_) * P.W + qw1_) * P.dq_ld + T.head * P.d;
#pragma unroll
    for (int j = 0; j < kTPW; ++j) {
      const int nt = nt0 + j;
      if (nt >= nt1) continue;
      if (v0) *reinterpret_cast<__nv_bfloat162*>(o0 + nt * 8 + 2 * t4) = __floats2bfloat162_rn(oq[j][0], oq[j][1]);
      if (v1) *reinterpret_cast<__nv_bfloat162*>(o1 + nt * 8 + 2 * t4) = __floats2bfloat162_rn(oq[j][2], oq[j][3]);
    }
  }
  if (qvalid) {
    float* drow = P.doffsets + (static_cast<long long>(T.b) * P.Nq + qrow) * P.doff_ld + static_cast<long long>(T.head) * K3;
    for (int j = js; j < je; ++j) {
      const unsigned long long v = rec[j];
      float gt = 0.f, gh = 0.f, gw = 0.f;
      if (v >> 63) {  // d p / d grid = S/2 strictly inside the volume, 0 on or beyond the border
        gt = ((v >> kBitInT) & 1ull) ? g3[3 * j + 0] * (0.5f * static_cast<float>(P.T)) : 0.f;
        gh = ((v >> kBitInH) & 1ull) ? g3[3 * j + 1] * (0.5f * static_cast<float>(P.H)) : 0.f;
        gw = ((v >> kBitInW) & 1ull) ? g3[3 * j + 2] * (0.5f * static_cast<float>(P.W)) : 0.f;
      }
      // offset channel 0 moved grid x (W) after division by (T-1), channel 1 grid y (H) by (H-1),
      // channel 2 grid z (T) by (W-1)
      drow[3 * j + 0] = P.T > 1 ? __fdiv_rn(gw, static_cast<float>(P.T - 1)) * P.oscale : 0.f;
      drow[3 * j + 1] = P.H > 1 ? __fdiv_rn(gh, static_cast<float>(P.H - 1)) * P.oscale : 0.f;
      drow[3 * j + 2] = P.W > 1 ? __fdiv_rn(gt, static_cast<float>(P.W - 1)) * P.oscale : 0.f;
    }
  }
}

}  // namespace bwd
}  // namespace tc

// ------------------------------------------------------------------------------ host side
bool tc_bwd_supported(const AttnParams& P) {
  if (!tc_supported(P)) return false;
  if (P.G != 0 || P.probs == nullptr) return false;
  return true;
}

bool tc_bwd_plan(const AttnParams& P, TcLaunch& L, int smem_limit) {
  const int dch = P.d / 8;
  L.rs = (dch & 1) ? P.d : P.d + 8;  // odd number of 16-byte chunks per row: conflict-free ldmatrix
  L.tiles_h = (P.H + tc::bwd::kTileH - 1) / tc::bwd::kTileH;
  L.tiles_w = (P.W + tc::kTileW - 1) / tc::kTileW;
  const size_t fixed = tc::bwd::smem_fixed(P, L.rs);
  const size_t per_key = static_cast<size_t>(L.rs) * 2 + static_cast<size_t>(tc::bwd::kQ) * 4;
  const size_t slack = static_cast<size_t>(tc::bwd::kQ) * 8 * 4;  // score-row padding (sld = maxkeys + 8)
  if (fixed + slack + per_key * 64 > static_cast<size_t>(smem_limit)) return false;
  int mk = static_cast<int>((static_cast<size_t>(smem_limit) - fixed - slack) / per_key);
  mk &= ~15;
  if (mk < 64) return false;
  if (mk > 1024) mk = 1024;
  L.maxkeys = mk;
  L.sld = mk + 8;  // row stride = 8 or 24 (mod 32) words: mma fragment rows hit distinct banks
  // the setup stages 32 queries x K x 3 offsets in the key buffer + score rows
  if (static_cast<size_t>(mk) * L.rs * 2 + static_cast<size_t>(tc::bwd::kQ) * L.sld * 4 <
      static_cast<size_t>(tc::bwd::kQ) * P.K * 12)
    return false;
  L.smem = static_cast<size_t>(mk) * L.rs * 2 + static_cast<size_t>(tc::bwd::kQ) * L.sld * 4 + fixed;
  L.tiles = static_cast<long long>(P.B) * P.q_frames * L.tiles_h * L.tiles_w * P.nh;
  return L.tiles <= 0x7fffffffLL && L.smem <= static_cast<size_t>(smem_limit);
}

template <int DCH>
static cudaError_t launch_bwd_tc_t(const AttnParams& P, const TcLaunch& L, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(tc::bwd::dsa_bwd_tc_kernel<DCH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  tc::bwd::dsa_bwd_tc_kernel<DCH><<<static_cast<unsigned>(L.tiles), tc::kThreads, L.smem, s>>>(P, L);
  return cudaGetLastError();
}

cudaError_t launch_attn_bwd_tc(const AttnParams& P, const TcLaunch& L, cudaStream_t s) {
  switch (P.d / 8) {
    case 2: return launch_bwd_tc_t<2>(P, L, s);
    case 3: return launch_bwd_tc_t<3>(P, L, s);
    case 4: return launch_bwd_tc_t<4>(P, L, s);
    case 5: return launch_bwd_tc_t<5>(P, L, s);
    case 6: return launch_bwd_tc_t<6>(P, L, s);
    case 7: return launch_bwd_tc_t<7>(P, L, s);
    case 8: return launch_bwd_tc_t<8>(P, L, s);
    case 9: return launch_bwd_tc_t<9>(P, L, s);
    case 10: return launch_bwd_tc_t<10>(P, L, s);
    case 11: return launch_bwd_tc_t<11>(P, L, s);
    case 12: return launch_bwd_tc_t<12>(P, L, s);
    case 13: return launch_bwd_tc_t<13>(P, L, s);
    case 14: return launch_bwd_tc_t<14>(P, L, s);
    case 15: return launch_bwd_tc_t<15>(P, L, s);
    case 16: return launch_bwd_tc_t<16>(P, L, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace msl
