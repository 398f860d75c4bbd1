// Tensor-core ("key envelope") backward of the deformable gather attention, bf16, no extra keys.
//
// One CTA owns a tile of 4 x 8 queries of one frame, one head and one sample (32 queries = two
// 16-query row groups; 16 warps, 8 per group; 16 lanes per query for the per-sample work).  Besides
// the forward's inputs it reads dO (gradient of the attention output), the forward output O and the
// forward's per-sample softmax weights p (`probs`).  With D = dO . O per query and, per window sample
// j with trilinear corners c and weights w_c, pv_j = p_j * keep_j / (1 - p_drop):
//
//   pass 1, per envelope chunk (V side):  dP = dO . V_chunk^T on the tensor cores; every sample adds
//            dp_j  += sum_c w_c dP[q, c]                   (dp_j = dO . v_j, before dropout)
//            gv_j  += sum_c (dw_c / dpix) dP[q, c]         (coordinate gradient, value part / pv_j)
//   then     dsq_j = softmax_scale * p_j * (keep_j dp_j / (1 - p_drop) - D),  g_j = pv_j gv_j
//   pass 2, per envelope chunk (K side):  S = Q . K_chunk^T; every sample adds
//            g_j   += dsq_j * sum_c (dw_c / dpix) S[q, c]  (coordinate gradient, key part)
//            and scatters dsq_j w_c into dS~[q, key] and pv_j w_c into P~[q, key];
//            dQ += dS~ . K_chunk,  dK_chunk = dS~^T . Q,  dV_chunk = P~^T . dO  (tensor cores)
//   dK / dV chunks are added to the float32 accumulators with vector atomics (one per 4 channels of
//   a key that received anything); g_j becomes the offset gradient through grid_sample's clip rule
//   and the offset normalisation, with the reference's axis swap.
//
// Per-sample work is spread over the whole CTA: the setup sorts the active samples into one list by
// frame (counting sort), so the samples with a corner in a plane are one contiguous range that all
// 512 threads stride through.  The setup also records, per (plane, chunk), which 16-key tiles any
// corner touches; loads, dense products and flushes visit only those tiles.  dS~ and P~ are
// accumulated with 32-bit integer shared atomics in fixed point (scale 2^21 / sum_j |value_j| per
// query, so no entry can overflow) and converted once per chunk into a transposed bf16 tile
// [key][query] that every product reads with ldmatrix.
//
// Reference semantics: autograd of infinity/video/attention.py:113-186 (grid_sampler_3d_backward,
// bmm and softmax backward, dropout).

#include "dsa_tc.cuh"

namespace msl {
namespace tc {
namespace bwd {

using namespace t32;



struct Smem {
  __nv_bfloat16* kbuf;      // [maxkeys][rs]   K or V chunk (setup: staged offsets, spilling into sa)
  float* sa;                // [32][sld]       dP / S (fp32), then P~ (int32), then P~^T (bf16 [key][40])
  float* sb;                // [32][sld]       dS~ (int32), then dS~^T (bf16 [key][40])
  __nv_bfloat16* qs;        // [32][rs]        Q rows of the tile
  __nv_bfloat16* dos;       // [32][rs]        dO rows of the tile
  unsigned long long* rec;  // [32][K]         packed sample records
  float* sv;                // [32][K]         dp_j, then dsq_j
  float* g3;                // [32][K][3]      coordinate gradient (t, h, w) before the clip rule
  int* key_off;             // [maxkeys]       row of each chunk key in the K/V buffers, -1 = none
  int* env;                 // envelope + base-grid tables
  float* dd;                // [32]            D = dO . O
  float* qsc;               // [4][32]         fixed-point scale / inverse of dS~ and P~ rows
  long long* prow;          // [32]            row of each query's softmax weights in probs
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
  s.sa = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * L.sld * 4;
  s.sb = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * L.sld * 4;
  s.qs = reinterpret_cast<__nv_bfloat16*>(base + off);
  off += static_cast<size_t>(kQ) * L.rs * 2;
  s.dos = reinterpret_cast<__nv_bfloat16*>(base + off);
  off += static_cast<size_t>(kQ) * L.rs * 2;
  s.rec = reinterpret_cast<unsigned long long*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 8;
  s.prow = reinterpret_cast<long long*>(base + off);
  off += kQ * 8;
  s.sv = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 4;
  s.g3 = reinterpret_cast<float*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 12;
  s.key_off = reinterpret_cast<int*>(base + off);
  off += static_cast<size_t>(L.maxkeys) * 4;
  s.env = reinterpret_cast<int*>(base + off);
  off += 16 * 4;  // envelope (the backward reads the forward's; no base-grid tables)
  s.dd = reinterpret_cast<float*>(base + off);
  off += kQ * 4;
  s.qsc = reinterpret_cast<float*>(base + off);
  off += 4 * kQ * 4;
  s.bstart = reinterpret_cast<int*>(base + off);
  off += (kBuckets + 4) * 4;
  s.bcur = reinterpret_cast<int*>(base + off);
  off += kBuckets * 4;
  s.mask = reinterpret_cast<uint32_t*>(base + off);
  off += 32 * kMaxMaskChunks * 4;
  s.hits = reinterpret_cast<unsigned short*>(base + off);
  off += static_cast<size_t>(kQ) * P.K * 2;
  off = (off + 7) & ~static_cast<size_t>(7);
  s.kbar = reinterpret_cast<unsigned long long*>(base + off);
  s.dead = reinterpret_cast<int*>(base + off + 8);
  return s;
}

// shared memory besides the key buffer, the two dense tiles and the key table
size_t smem_fixed(const AttnParams& P, int rs) {
  return static_cast<size_t>(kQ) * rs * 2 * 2 + static_cast<size_t>(kQ) * P.K * (8 + 4 + 12 + 2) + 16 * 4 +
         kQ * (8 + 4 + 16) + (2 * kBuckets + 4 + 32 * kMaxMaskChunks) * 4 + 24 + 256;
}

// In-plane terms of one sample from a dense row (corners outside the volume count as 0, like
// grid_sample's zero contribution of out-of-bounds corners):
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
  t.bil = ay0 * fmaf(ax1, v01, ax0 * v00) + ay1 * fmaf(ax1, v11, ax0 * v10);
  t.dvx = ay0 * (v01 - v00) + ay1 * (v11 - v10);
  t.dvy = ax0 * (v10 - v00) + ax1 * (v11 - v01);
  return t;
}


constexpr int kDqChannelGroups = 4;  // dQ product: channel ranges per row group (x 2 key-tile parts)

// ------------------------------------------------------------------------------ chunk operands
// accum[key][d] += A . X over the tiles of mask m: A = the transposed bf16 tile tb ([key][query], all
// 32 queries, ldmatrix), X = 32 bf16 rows (Q or dO) in shared memory.  Items = (16-key tile, the
// head's channel tiles when their count is odd and at most 9, else half of them), round robin over
// the 16 warps: one A fragment serves every accumulator chain of the item (measured: at head_dim 72
// whole-head items beat 3 or 5 channel tiles; at head_dim 64 half-head items beat whole-head ones,
// the warps get twice the items).  Each lane adds its fragment pairs to the float32 accumulator rows
// key_off[key] with float2 atomics, skipping the rows of keys no sample corner touched (all zero).
template <int DCH>
__device__ __forceinline__ void kv_product_flush(const AttnParams& P, const TileCtx& T, const TcLaunch& L,
                                                 const __nv_bfloat16* tb, const __nv_bfloat16* xs, const int* key_off,
                                                 uint32_t m, float* accum) {
  constexpr int NG = (DCH & 1) && DCH <= 9 ? DCH : (DCH + 1) / 2;  // channel tiles per item (head or half)
  constexpr int NCG = (DCH + NG - 1) / NG;  // channel groups
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  const int items = __popc(m) * NCG;
  float* const abase = accum + static_cast<long long>(T.b) * P.Nkv * P.acc_ld + T.head * P.d + 2 * t4;
  const int tl = nth_bit(m, lane);  // lane o: the o-th touched tile (one bit search per warp)
  for (int item = warp; item < items; item += kWarps) {
    const int mo = item / NCG, cg = item - mo * NCG;
    const int tile = __shfl_sync(kFull, tl, mo);
    const int nt0 = cg * NG;
    float c[NG][4];
#pragma unroll
    for (int j = 0; j < NG; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t a[4];  // rows = keys tile*16 + 0..15, columns = queries kk*16 + 0..15
      ldsm_x4(smem_u32(tb + static_cast<size_t>(tile * 16 + (lane & 15)) * kTRow + kk * 16 + (lane >> 4) * 8), a[0], a[1],
              a[2], a[3]);
      // x4.trans matrices: (queries +0..7, ch nt) (queries +8..15, ch nt) (+0..7, nt+1) (+8..15, nt+1)
      const __nv_bfloat16* rowp = xs + static_cast<size_t>(kk * 16 + rr + ((mi & 1) ? 8 : 0)) * L.rs;
#pragma unroll
      for (int j = 0; j < NG; j += 2) {
        if (nt0 + j + 1 < DCH && j + 1 < NG) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(rowp + (nt0 + j + (mi >> 1)) * 8), b0, b1, b2, b3);
          mma16816(c[j], a, b0, b1);
          mma16816(c[j + 1], a, b2, b3);
        } else if (nt0 + j < DCH) {
          uint32_t b0, b1;
          ldsm_x2_t(smem_u32(rowp + (nt0 + j) * 8), b0, b1);
          mma16816(c[j], a, b0, b1);
        }
      }
    }
    const int o0 = key_off[tile * 16 + g], o1 = key_off[tile * 16 + g + 8];
    float* const a0 = abase + static_cast<long long>(max(o0, 0)) * P.acc_ld + nt0 * 8;
    float* const a1 = abase + static_cast<long long>(max(o1, 0)) * P.acc_ld + nt0 * 8;
    // a key no sample corner touched has an all-zero row (about a fifth of the flushed keys): its
    // accumulator row is skipped (the four lanes of a row agree through two shuffles)
    bool nz0 = false, nz1 = false;
#pragma unroll
    for (int j = 0; j < NG; ++j) {
      if (nt0 + j >= DCH) break;
      nz0 |= (c[j][0] != 0.f) | (c[j][1] != 0.f);
      nz1 |= (c[j][2] != 0.f) | (c[j][3] != 0.f);
    }
    const int nzb = (nz0 ? 1 : 0) | (nz1 ? 2 : 0);
    const int nzr = nzb | __shfl_xor_sync(kFull, nzb, 1) | __shfl_xor_sync(kFull, nzb, 2) |
                    __shfl_xor_sync(kFull, nzb, 3);
    const bool w0 = o0 >= 0 && (nzr & 1), w1 = o1 >= 0 && (nzr & 2);
#pragma unroll
    for (int j = 0; j < NG; ++j) {
      if (nt0 + j >= DCH) break;  // warp-uniform
      // the fragment's own pairs: key g (c0, c1) and key g + 8 (c2, c3), channels 8 (nt0 + j) + 2t4, +1
      if (w0) atomicAdd(reinterpret_cast<float2*>(a0 + j * 8), make_float2(c[j][0], c[j][1]));
      if (w1) atomicAdd(reinterpret_cast<float2*>(a1 + j * 8), make_float2(c[j][2], c[j][3]));
    }
  }
}

template <int DCH>
__global__ void __launch_bounds__(kThreads, 1) dsa_bwd_tc_kernel(const AttnParams P, const TcLaunch L,
                                                                  const __grid_constant__ KeyMaps maps) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const Smem S = carve(smem_raw, P, L);
  const TileCtx T = decode_tile(P, L, kTileH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp / kWPG, part = warp - (warp / kWPG) * kWPG;
  const int ll = part * 32 + lane;
  const int cq = ll / kLPQ, sub = ll - (ll / kLPQ) * kLPQ;
  const int K = P.K;
  // setup and final stores: the lanes of a query own contiguous window ranges [js, je)
  const int jper = (K + kLPQ - 1) / kLPQ;
  const int js = min(K, sub * jper), je = min(K, js + jper);
  const int n = je - js;       // samples of this lane
  const int qi = r * 16 + cq;  // owned query within the tile
  const float invK = 1.f / static_cast<float>(K);

  int qh, qw;
  query_hw(T, r, cq, qh, qw);
  const bool qvalid = qh < P.H && qw < P.W;
  const long long qrow = (static_cast<long long>(T.tl) * P.H + qh) * P.W + qw;
  const int qbase = qi * K;  // this query's samples in rec / sv / g3

  if (threadIdx.x < kBuckets) S.bcur[threadIdx.x] = 0;
  if (threadIdx.x < 32 * kMaxMaskChunks) S.mask[threadIdx.x] = 0u;
  if (sub == 0) S.prow[qi] = (static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow;
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

  // ---- stage the forward's records of the tile (this head), Q and dO rows with one wave of cp.async;
  //      the tile's envelope as the forward computed it
  const unsigned long long* recs = static_cast<const unsigned long long*>(P.saved);
  for (int q2 = warp; q2 < kQ; q2 += kWarps) {
    int sqh, sqw;
    query_hw(T, q2 >> 4, q2 & 15, sqh, sqw);
    const bool ok = sqh < P.H && sqw < P.W;
    const long long prow = (static_cast<long long>(T.tl) * P.H + sqh) * P.W + sqw;
    const long long grow = static_cast<long long>(T.b) * P.Nq + prow;
    unsigned long long* rdst = S.rec + static_cast<size_t>(q2) * K;
    if (ok) {
      const unsigned long long* src = recs + ((static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + prow) * K;
      for (int k = lane; k < K; k += 32) cp_async8(smem_u32(rdst + k), src + k);
    } else {
      for (int k = lane; k < K; k += 32) rdst[k] = 0ull;
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
  if (threadIdx.x < 6) S.env[threadIdx.x] =
      reinterpret_cast<const int*>(static_cast<const char*>(P.saved) + saved_env_offset(P))[8 * blockIdx.x + threadIdx.x];
  cp_async_wait_all();
  __syncthreads();

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
  if (overflow) return;  // the forward computed this tile with the CUDA-core gather: so does
                         // dsa_bwd_tc_fallback_kernel (no copy was issued yet)
  const bool work = any && !overflow;
  const bool masks = work && E.ny * E.nx <= kMaxMaskChunks;
  const bool fsplit = split && !masks;  // chunks of a plane share one hit bucket: filter the hits
  // pass 1's first V chunk (plane zlo, chunk 0, every tile of it) loads while the setup runs
  const bool early = tma && work;
  if (early) {
    Chunk k0;
    k0.zr = k0.iy = k0.ix = 0;
    k0.m = chunk_mask(E, S.mask, false, k0);
    if (!*S.dead) issue_keys_tma(P, T, E, k0, S.kbuf, L.rs, maps.v, maps.have, kbar, true);
  }

  // ---- the forward's records with this kernel's chunk bits; frame-bucket counts and touched-tile masks
  for (int s = 0; s < jper; ++s) {
    const int j = js + s;
    int bk = -1, pa = -1, pb = -1;
    uint32_t bits = 0u;
    if (qvalid && s < n) {
      unsigned long long v = S.rec[qbase + j];
      if (!work) v = 0ull;
      if (v >> 63) {  // a corner in a frame the K/V buffers hold
        const int dz = static_cast<int>((v >> 36) & 0x1fu);
        const int t0 = E.zlo - 1 + dz, h0 = E.ylo + static_cast<int>((v >> 41) & 0xffu),
                  w0 = E.xlo + static_cast<int>((v >> 49) & 0xffu);
        v &= ~(3ull << kBitChunk);
        bk = dz;
        if (masks) {
          const int iy = axis_chunk_of(h0, E.ylo, E.R, E.ny), ix = axis_chunk_of(w0, E.xlo, E.cw, E.nx);
          const int ya = E.ylo + iy * (E.R - 1), xa = E.xlo + ix * (E.cw - 1);
          bits = corner_tiles((h0 - ya) * E.kst + (w0 - xa), E.kst, w0 + 1 < P.W, h0 + 1 < P.H);
          const int chk = iy * E.nx + ix;
          if (t0 >= E.zlo) pa = dz * kMaxMaskChunks + chk;           // plane z = t0 (zrel = dz)
          if (t0 + 1 <= E.zhi) pb = (dz + 1) * kMaxMaskChunks + chk; // plane z = t0 + 1
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
  __syncthreads();
  if (warp == 0) scan_buckets(S.bcur, S.bstart);
  __syncthreads();
  // hit list: every active sample once, grouped by (chunk, frame) bucket
  for (int s = 0; s < jper; ++s) {
    const int j = js + s;
    int bk = -1;
    if (qvalid && s < n) {
      const unsigned long long v = S.rec[qbase + j];
      if (v >> 63) bk = rec_bucket(v);
      S.sv[qbase + j] = 0.f;
      S.g3[3 * (qbase + j)] = 0.f;
      S.g3[3 * (qbase + j) + 1] = 0.f;
      S.g3[3 * (qbase + j) + 2] = 0.f;
    }
    if (bk >= 0) S.hits[atomicAdd(S.bcur + bk, 1)] = static_cast<unsigned short>(qbase + j);
  }

  const int g = lane >> 2, t4 = lane & 3;
  float* grow_a = S.sa + static_cast<size_t>(r) * 16 * L.sld;  // the row group's 16 dense rows
  __syncthreads();

  // ---- pass 1: V side (dp_j and the value part of the coordinate gradient), hits CTA-wide; the next
  // chunk's values load while this chunk's samples run, and after the last one pass 2's first keys
  const int nz = work ? E.zhi - E.zlo + 1 : 0;
  const __nv_bfloat16* kg = static_cast<const __nv_bfloat16*>(P.k);
  const __nv_bfloat16* vg = static_cast<const __nv_bfloat16*>(P.v);
  const int kst = E.kst;
  Chunk k2;  // pass 2's first chunk
  const bool have2 = chunk_first(E, S.mask, masks, nz, k2);
  {
    Chunk k = k2;
    bool have = have2;
    if (early && !(have && k.zr == 0 && k.iy == 0 && k.ix == 0)) {
      // the early chunk is not the walk's first: let its copies land before the buffer is reused
      wait_keys(kbar, kphase, S.dead, P.status);
      kphase ^= 1u;
      __syncthreads();
    }
    if (have && !(early && k.zr == 0 && k.iy == 0 && k.ix == 0)) {
      if (tma) {
        if (!*S.dead) issue_keys_tma(P, T, E, k, S.kbuf, L.rs, maps.v, maps.have, kbar, !early);
      } else {
        issue_keys<DCH>(P, T, E, k, S.kbuf, L.rs, vg, P.v_ld);
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
      dense_tiles<DCH, kWPG>(S.kbuf, S.dos + static_cast<size_t>(r) * 16 * L.rs, L.rs, grow_a, L.sld, part, cur.m);
      __syncthreads();
      have = chunk_next(E, S.mask, masks, nz, k);
      const bool v = have;
      if (!have) k = k2;
      if (tma) {
        if (!*S.dead) issue_keys_tma(P, T, E, k, S.kbuf, L.rs, v ? maps.v : maps.k, maps.have, kbar, false);
      } else {
        issue_keys<DCH>(P, T, E, k, S.kbuf, L.rs, v ? vg : kg, v ? P.v_ld : P.k_ld);
      }
      const int z = E.zlo + cur.zr, ya = chunk_ya(E, cur), xa = chunk_xa(E, cur);
      const int hb = (masks ? cur.iy * E.nx + cur.ix : 0) * 32 + cur.zr;
      const int hlo = S.bstart[hb], hhi = S.bstart[hb + 2];
      for (int i = hlo + static_cast<int>(threadIdx.x); i < hhi; i += kThreads) {
        const int idx = S.hits[i];
        const int q = static_cast<int>((static_cast<float>(idx) + 0.5f) * invK);
        const Rec rc = decode_rec(S.rec[idx], E);
        if (fsplit && (axis_chunk_of(rc.h0, E.ylo, E.R, E.ny) != cur.iy || axis_chunk_of(rc.w0, E.xlo, E.cw, E.nx) != cur.ix))
          continue;
        const bool upper = z != rc.t0;
        const float az = frac_weight(rc.ft, upper);
        const PlaneTerms pt_ =
            plane_terms(S.sa + static_cast<size_t>(q) * L.sld, (rc.h0 - ya) * kst + (rc.w0 - xa), kst, rc, P.H, P.W);
        S.sv[idx] = fmaf(az, pt_.bil, S.sv[idx]);
        float* gg = S.g3 + 3 * idx;
        gg[0] += upper ? pt_.bil : -pt_.bil;
        gg[1] = fmaf(az, pt_.dvy, gg[1]);
        gg[2] = fmaf(az, pt_.dvx, gg[2]);
      }
    }
  }
  __syncthreads();

  // ---- dsq_j = softmax_scale * p_j * (keep_j dp_j / (1 - p_drop) - D); g_j = pv_j gv_j; row scales
  {
    float bds = 0.f, bp = 0.f;
    if (qvalid) {
      const float D = S.dd[qi];
      const float* prob_row = P.probs + S.prow[qi] * K;
      for (int j = js; j < je; ++j) {
        const unsigned long long v = S.rec[qbase + j];
        if (!(v >> 63)) continue;
        const float p = __ldg(prob_row + j);
        const bool keep = (v >> kBitKeep) & 1ull;
        const float pv = keep ? p * P.drop_keep_scale : 0.f;
        const float kf = keep ? P.drop_keep_scale : 0.f;
        const float dsq = p * fmaf(kf, S.sv[qbase + j], -D) * P.scale;
        S.sv[qbase + j] = dsq;
        float* gg = S.g3 + 3 * (qbase + j);
        gg[0] *= pv;
        gg[1] *= pv;
        gg[2] *= pv;
        bds += fabsf(dsq);
        bp += pv;
      }
    }
#pragma unroll
    for (int o = 1; o < kLPQ; o <<= 1) {
      bds += __shfl_xor_sync(kFull, bds, o);
      bp += __shfl_xor_sync(kFull, bp, o);
    }
    if (sub == 0) {
      S.qsc[qi] = bds > 0.f ? kFixRange / bds : 1.f;
      S.qsc[kQ + qi] = bds > 0.f ? bds / kFixRange : 0.f;
      S.qsc[2 * kQ + qi] = bp > 0.f ? kFixRange / bp : 1.f;
      S.qsc[3 * kQ + qi] = bp > 0.f ? bp / kFixRange : 0.f;
    }
  }
  __syncthreads();

  // ---- pass 2: K side (key part of the coordinate gradient, dQ, dK, dV), hits CTA-wide
  // dQ: the 8 warps of a row group = kCG channel ranges x kKS parts of the touched key tiles (measured
  // at head_dim 72: 4 x 2 beats 8 x 1 and 2 x 4)
  constexpr int kCG = kDqChannelGroups, kKS = kWPG / kCG;
  constexpr int kCB = DCH / kCG, kCX = DCH % kCG;
  constexpr int kTPW = kCB + (kCX ? 1 : 0);  // dQ channel tiles per warp (at most)
  const int cpart = part % kCG, kpar = part / kCG;
  const int nt0 = cpart * kCB + min(cpart, kCX), nt1 = nt0 + kCB + (cpart < kCX ? 1 : 0);
  float oq[kTPW + 1][4];
#pragma unroll
  for (int i = 0; i < kTPW + 1; ++i) oq[i][0] = oq[i][1] = oq[i][2] = oq[i][3] = 0.f;
  const __nv_bfloat16* tds = reinterpret_cast<const __nv_bfloat16*>(S.sb);  // dS~^T after the transposition
  const __nv_bfloat16* tpp = reinterpret_cast<const __nv_bfloat16*>(S.sa);  // P~^T after the transposition
  // (the first chunk's keys were issued at the end of pass 1; each later chunk's keys load while the
  // previous chunk's P~ is converted and its dV flushed)
  {
    Chunk k = k2;
    bool have = have2;
    while (have) {
      const Chunk cur = k;
      const int z = E.zlo + cur.zr, ya = chunk_ya(E, cur), xa = chunk_xa(E, cur);
      const int hb = (masks ? cur.iy * E.nx + cur.ix : 0) * 32 + cur.zr;
      const int hlo = S.bstart[hb], hhi = S.bstart[hb + 2];
      if (tma) {
        wait_keys(kbar, kphase, S.dead, P.status);
        kphase ^= 1u;
      } else {
        cp_async_wait_all();
      }
      __syncthreads();  // keys landed; the previous chunk's dV flush is done with key_off and sa
      if (tma && tile_dead(S.dead)) break;  // a wait gave up: nothing more reads the key buffer
      for (int i = threadIdx.x; i < __popc(cur.m) * 16; i += kThreads) {
        const int key = nth_bit(cur.m, i >> 4) * 16 + (i & 15);
        S.key_off[key] = chunk_key_row(P, E, cur, key);
      }
      zero_tiles<kQ>(S.sb, L.sld, cur.m);
      dense_tiles<DCH, kWPG>(S.kbuf, S.qs + static_cast<size_t>(r) * 16 * L.rs, L.rs, grow_a, L.sld, part, cur.m);
      __syncthreads();
      // key part of the coordinate gradient (reads S) and the dS~ scatter (into sb)
      for (int i = hlo + static_cast<int>(threadIdx.x); i < hhi; i += kThreads) {
        const int idx = S.hits[i];
        const int q = static_cast<int>((static_cast<float>(idx) + 0.5f) * invK);
        const Rec rc = decode_rec(S.rec[idx], E);
        if (fsplit && (axis_chunk_of(rc.h0, E.ylo, E.R, E.ny) != cur.iy || axis_chunk_of(rc.w0, E.xlo, E.cw, E.nx) != cur.ix))
          continue;
        const bool upper = z != rc.t0;
        const float az = frac_weight(rc.ft, upper);
        const int k00 = (rc.h0 - ya) * kst + (rc.w0 - xa);
        const PlaneTerms pt_ = plane_terms(S.sa + static_cast<size_t>(q) * L.sld, k00, kst, rc, P.H, P.W);
        const float dsq = S.sv[idx];
        float* gg = S.g3 + 3 * idx;
        gg[0] = fmaf(dsq, upper ? pt_.bil : -pt_.bil, gg[0]);
        gg[1] = fmaf(dsq * az, pt_.dvy, gg[1]);
        gg[2] = fmaf(dsq * az, pt_.dvx, gg[2]);
        scatter_fixed_row(reinterpret_cast<int*>(S.sb) + static_cast<size_t>(q) * L.sld, k00, kst, rc,
                          dsq * az * S.qsc[q], P.H, P.W);
      }
      __syncthreads();
      // dS~ -> bf16 [key][query]; S no longer needed: clear sa for P~
      transpose_fixed<kMaxKeys>(S.sb, L.sld, cur.m, S.qsc + kQ);
      zero_tiles<kQ>(S.sa, L.sld, cur.m);
      __syncthreads();
      // P~ scatter (into sa), dQ += dS~ . K_chunk, dK_chunk = dS~^T . Q
      // two hits per step, their softmax weights loaded first (global loads: overlap their latency)
      for (int i = hlo + static_cast<int>(threadIdx.x); i < hhi; i += 2 * kThreads) {
        const int i1 = i + kThreads;
        const bool two = i1 < hhi;
        const int idx0 = S.hits[i], idx1 = two ? S.hits[i1] : idx0;
        const int q0 = static_cast<int>((static_cast<float>(idx0) + 0.5f) * invK);
        const int q1 = static_cast<int>((static_cast<float>(idx1) + 0.5f) * invK);
        const float p0 = __ldg(P.probs + S.prow[q0] * K + (idx0 - q0 * K));
        const float p1 = two ? __ldg(P.probs + S.prow[q1] * K + (idx1 - q1 * K)) : 0.f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (u == 1 && !two) break;
          const int idx = u ? idx1 : idx0, q = u ? q1 : q0;
          const unsigned long long v = S.rec[idx];
          if (!((v >> kBitKeep) & 1ull)) continue;
          const Rec rc = decode_rec(v, E);
          if (fsplit && (axis_chunk_of(rc.h0, E.ylo, E.R, E.ny) != cur.iy || axis_chunk_of(rc.w0, E.xlo, E.cw, E.nx) != cur.ix))
            continue;
          const float pv = (u ? p1 : p0) * P.drop_keep_scale;
          scatter_fixed_row(reinterpret_cast<int*>(S.sa) + static_cast<size_t>(q) * L.sld,
                            (rc.h0 - ya) * kst + (rc.w0 - xa), kst, rc,
                            pv * frac_weight(rc.ft, z != rc.t0) * S.qsc[2 * kQ + q], P.H, P.W);
        }
      }
      dq_product<DCH, kTPW, kKS>(tds, r, S.kbuf, L.rs, nt0, nt1, cur.m, oq, kpar);
      kv_product_flush<DCH>(P, T, L, tds, S.qs, S.key_off, cur.m, P.dk_acc);
      __syncthreads();  // the key buffer is free
      have = chunk_next(E, S.mask, masks, nz, k);
      if (have) {
        if (tma) {
          if (!*S.dead) issue_keys_tma(P, T, E, k, S.kbuf, L.rs, maps.k, maps.have, kbar, false);
        } else {
          issue_keys<DCH>(P, T, E, k, S.kbuf, L.rs, kg, P.k_ld);
        }
      }
      transpose_fixed<kMaxKeys>(S.sa, L.sld, cur.m, S.qsc + 3 * kQ);
      __syncthreads();
      kv_product_flush<DCH>(P, T, L, tpp, S.dos, S.key_off, cur.m, P.dv_acc);
    }
  }
  __syncthreads();

  // ---- extra keys / values shared by every query of the sample (attention.py:159-173): dO . EV^T and
  //      Q . EK^T on the tensor cores, the softmax weights from the forward's log-sum-exp; every
  //      (query, extra key) dS and weight goes to extra_ds / extra_p (dsa_extra_grad_kernel reduces them
  //      over the queries into d(ek), d(ev)), and dQ += dS_extra . EK on the tensor cores
  if (P.G > 0 && !(tma && tile_dead(S.dead))) {
    const int gp = (P.G + 15) & ~15;
    const uint32_t gmask = gp >= 512 ? 0xffffffffu : (1u << (gp >> 4)) - 1u;
    load_extra<DCH>(P, T, S.kbuf, L.rs, P.ev, gp);
    __syncthreads();
    dense_tiles<DCH, kWPG>(S.kbuf, S.dos + static_cast<size_t>(r) * 16 * L.rs, L.rs,
                           S.sb + static_cast<size_t>(r) * 16 * L.sld, L.sld, part, gmask);
    __syncthreads();
    load_extra<DCH>(P, T, S.kbuf, L.rs, P.ek, gp);
    __syncthreads();
    dense_tiles<DCH, kWPG>(S.kbuf, S.qs + static_cast<size_t>(r) * 16 * L.rs, L.rs, grow_a, L.sld, part, gmask);
    __syncthreads();
    if (qvalid) {  // dS in place of dP: each element is read and written by one thread
      const float lse2 = P.lse[(static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow];
      const float dq_d = S.dd[qi];
      const uint64_t qg = ((static_cast<uint64_t>(T.b) * P.T + T.tg) * P.H + qh) * P.W + qw;
      const long long xrow = ((static_cast<long long>(T.b) * P.nh + T.head) * P.Nq + qrow) * P.G;
      for (int e = sub; e < P.G; e += kLPQ) {
        const float p = exp2f(S.sa[static_cast<size_t>(qi) * L.sld + e] * P.scale_log2 - lse2);
        float ks = 1.f;
        if (P.drop_thresh)
          ks = dropout_keep(P.seed, (qg * P.nh + T.head) * static_cast<uint64_t>(K + P.G) + K + e, P.drop_thresh)
                   ? P.drop_keep_scale
                   : 0.f;
        float* dpe = S.sb + static_cast<size_t>(qi) * L.sld + e;
        const float dsq = p * (*dpe * ks - dq_d) * P.scale;
        P.extra_ds[xrow + e] = dsq;
        P.extra_p[xrow + e] = p * ks;
        *dpe = dsq;
      }
    }
    __syncthreads();
    // dS_extra^T as a bf16 tile [key][query] in sa (zero for padding keys and queries outside the volume)
    __nv_bfloat16* te = reinterpret_cast<__nv_bfloat16*>(S.sa);
    for (int i = threadIdx.x; i < gp * kQ; i += kThreads) {
      const int e = i / kQ, q = i - (i / kQ) * kQ;
      int qh2, qw2;
      query_hw(T, q >> 4, q & 15, qh2, qw2);
      const bool ok = e < P.G && qh2 < P.H && qw2 < P.W;
      te[static_cast<size_t>(e) * kTRow + q] = __float2bfloat16_rn(ok ? S.sb[static_cast<size_t>(q) * L.sld + e] : 0.f);
    }
    __syncthreads();
    dq_product<DCH, kTPW, kKS>(te, r, S.kbuf, L.rs, nt0, nt1, gmask, oq, kpar);
    __syncthreads();
  }

  // ---- the warps of the other key-tile parts hand their dQ partial sums to part 0 (through the key
  //      buffer and the dense tiles, contiguous and free now: [2][kCG][kKS - 1][kTPW][32] float4)
  if (kKS > 1) {
    float4* red = reinterpret_cast<float4*>(S.kbuf) + ((r * kCG + cpart) * (kKS - 1) * kTPW) * 32 + lane;
    if (kpar > 0) {
#pragma unroll
      for (int j = 0; j < kTPW; ++j)
        if (nt0 + j < nt1) red[((kpar - 1) * kTPW + j) * 32] = make_float4(oq[j][0], oq[j][1], oq[j][2], oq[j][3]);
    }
    __syncthreads();
    if (kpar == 0) {
      for (int u = 0; u < kKS - 1; ++u) {
#pragma unroll
        for (int j = 0; j < kTPW; ++j) {
          if (nt0 + j >= nt1) continue;
          const float4 t = red[(u * kTPW + j) * 32];
          oq[j][0] += t.x;
          oq[j][1] += t.y;
          oq[j][2] += t.z;
          oq[j][3] += t.w;
        }
      }
    }
  }

  // ---- dQ (bf16) and the offset gradients
  if (kpar == 0) {
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
    const int K3 = 3 * K;
    const long long drow = (static_cast<long long>(T.b) * P.Nq + qrow) * P.doff_ld + static_cast<long long>(T.head) * K3;
    // d p / d grid = S/2 strictly inside the volume (0 on or beyond the border), times the offset
    // normalisation: channel 0 moved grid x (W) after division by (T-1), channel 1 grid y (H) by
    // (H-1), channel 2 grid z (T) by (W-1)
    const float c0 = P.T > 1 ? 0.5f * static_cast<float>(P.W) * P.oscale / static_cast<float>(P.T - 1) : 0.f;
    const float c1 = P.H > 1 ? 0.5f * static_cast<float>(P.H) * P.oscale / static_cast<float>(P.H - 1) : 0.f;
    const float c2 = P.W > 1 ? 0.5f * static_cast<float>(P.T) * P.oscale / static_cast<float>(P.W - 1) : 0.f;
    // element e = 3j + c of the row (the 16 lanes of the query store consecutive floats): channel c
    // takes coordinate gradient component 2 - c (w, h, t) and the interior flag of that axis
    for (int e = sub; e < K3; e += kLPQ) {
      const int j = e / 3, c = e - 3 * j;
      const unsigned long long v = S.rec[qbase + j];
      const float cc = c == 0 ? c0 : (c == 1 ? c1 : c2);
      const bool on = (v >> 63) && ((v >> (kBitInW - c)) & 1ull);
      store_doff(P, drow + e, on ? S.g3[3 * (qbase + j) + 2 - c] * cc : 0.f);
    }
  }
}

}  // namespace bwd
}  // namespace tc

// ------------------------------------------------------------------------------ host side
bool tc_bwd_supported(const AttnParams& P) {
  if (!tc_supported(P)) return false;
  if (P.probs == nullptr || P.saved == nullptr) return false;
  if (static_cast<long long>(tc::bwd::kQ) * P.K > 65536) return false;  // hit-list entries are 16-bit
  return true;
}

bool tc_bwd_plan(const AttnParams& P, TcLaunch& L, int smem_limit) {
  const int dch = P.d / 8;
  L.rs = (dch & 1) ? P.d : P.d + 8;  // odd number of 16-byte chunks per row: conflict-free ldmatrix
  L.tiles_h = (P.H + tc::bwd::kTileH - 1) / tc::bwd::kTileH;
  L.tiles_w = (P.W + tc::kTileW - 1) / tc::kTileW;
  const size_t fixed = tc::bwd::smem_fixed(P, L.rs);
  // per key: its K/V row, two dense fp32 columns, its key-table entry
  const size_t per_key = static_cast<size_t>(L.rs) * 2 + 2 * static_cast<size_t>(tc::bwd::kQ) * 4 + 4;
  const size_t slack = 2 * static_cast<size_t>(tc::bwd::kQ) * 8 * 4;  // dense-row padding (sld = maxkeys + 8)
  if (fixed + slack + per_key * 64 > static_cast<size_t>(smem_limit)) return false;
  int mk = static_cast<int>((static_cast<size_t>(smem_limit) - fixed - slack) / per_key);
  mk &= ~15;
  if (mk < 64) return false;
  if (mk > tc::bwd::kMaxKeys) mk = tc::bwd::kMaxKeys;
  if (((P.G + 15) & ~15) > mk) return false;  // the extra keys are one chunk of the key buffer
  L.maxkeys = mk;
  L.sld = mk + 8;  // row stride = 8 or 24 (mod 32) words: mma fragment rows hit distinct banks
  // a transposed bf16 tile [maxkeys][40] must fit in a dense fp32 tile [32][sld]
  if (static_cast<size_t>(mk) * tc::bwd::kTRow * 2 > static_cast<size_t>(tc::bwd::kQ) * L.sld * 4) return false;
  // the dQ partial sums handed between the key-tile parts fit the key buffer + the two dense tiles
  {
    const int cg = tc::bwd::kDqChannelGroups, ks = tc::bwd::kWPG / cg, tpw = (dch + cg - 1) / cg;
    if (static_cast<size_t>(2) * cg * (ks - 1) * tpw * 512 >
        static_cast<size_t>(mk) * L.rs * 2 + 2 * static_cast<size_t>(tc::bwd::kQ) * L.sld * 4)
      return false;
  }
  L.smem = static_cast<size_t>(mk) * L.rs * 2 + 2 * static_cast<size_t>(tc::bwd::kQ) * L.sld * 4 +
           static_cast<size_t>(mk) * 4 + fixed;
  L.tiles = static_cast<long long>(P.B) * P.q_frames * L.tiles_h * L.tiles_w * P.nh;
  return L.tiles <= 0x7fffffffLL && L.smem <= static_cast<size_t>(smem_limit);
}

namespace tc {
namespace bwd {
// The backward of the tiles the tensor-core kernels leave to the CUDA-core gather (key envelopes the
// sample records cannot encode: env_overflow on the forward's saved envelope).  A CTA checks 32
// consecutive tiles' envelopes (one per lane of warp 0) and runs the gather for those that overflow;
// in the common case every CTA exits after that one check.
constexpr int kFallbackWarps = 4;
constexpr int kFallbackTiles = 32;
template <int DCH>
__global__ void __launch_bounds__(32 * kFallbackWarps) dsa_bwd_tc_fallback_kernel(const AttnParams P, const TcLaunch L) {
  __shared__ uint32_t over;
  const long long t0 = static_cast<long long>(blockIdx.x) * kFallbackTiles;
  if (threadIdx.x < 32) {
    const long long t = t0 + threadIdx.x;
    bool o = false;
    if (t < L.tiles) {
      const int4* env = reinterpret_cast<const int4*>(static_cast<const char*>(P.saved) + saved_env_offset(P)) + 2 * t;
      const int4 a = env[0], b = env[1];
      o = env_overflow(a.x, a.y, a.z, a.w, b.x, b.y);
    }
    const uint32_t m = __ballot_sync(0xffffffffu, o);
    if (threadIdx.x == 0) over = m;
  }
  __syncthreads();
  for (uint32_t m = over; m; m &= m - 1u) {
    const long long tile = t0 + __ffs(m) - 1;
    const TileCtx T = decode_tile_index(P, L, kTileH, tile);
    tile_fallback<DCH, true, kFallbackWarps>(P, T);
  }
}
}  // namespace bwd
}  // namespace tc

template <int DCH>
static cudaError_t launch_bwd_tc_t(const AttnParams& P, const TcLaunch& L, const tc::KeyMaps& maps,
                                   cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(tc::bwd::dsa_bwd_tc_kernel<DCH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  tc::bwd::dsa_bwd_tc_kernel<DCH><<<static_cast<unsigned>(L.tiles), tc::kThreads, L.smem, s>>>(P, L, maps);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long nfb = (L.tiles + tc::bwd::kFallbackTiles - 1) / tc::bwd::kFallbackTiles;
  tc::bwd::dsa_bwd_tc_fallback_kernel<DCH><<<static_cast<unsigned>(nfb), 32 * tc::bwd::kFallbackWarps, 0, s>>>(P, L);
  return cudaGetLastError();
}

cudaError_t launch_attn_bwd_tc(const AttnParams& P, const TcLaunch& L0, cudaStream_t s) {
  TcLaunch L = L0;
  tc::KeyMaps maps;
  L.tma = tc::make_key_maps(&maps, P, L.rs);
  switch (P.d / 8) {
    case 2: return launch_bwd_tc_t<2>(P, L, maps, s);
    case 3: return launch_bwd_tc_t<3>(P, L, maps, s);
    case 4: return launch_bwd_tc_t<4>(P, L, maps, s);
    case 5: return launch_bwd_tc_t<5>(P, L, maps, s);
    case 6: return launch_bwd_tc_t<6>(P, L, maps, s);
    case 7: return launch_bwd_tc_t<7>(P, L, maps, s);
    case 8: return launch_bwd_tc_t<8>(P, L, maps, s);
    case 9: return launch_bwd_tc_t<9>(P, L, maps, s);
    case 10: return launch_bwd_tc_t<10>(P, L, maps, s);
    case 11: return launch_bwd_tc_t<11>(P, L, maps, s);
    case 12: return launch_bwd_tc_t<12>(P, L, maps, s);
    case 13: return launch_bwd_tc_t<13>(P, L, maps, s);
    case 14: return launch_bwd_tc_t<14>(P, L, maps, s);
    case 15: return launch_bwd_tc_t<15>(P, L, maps, s);
    case 16: return launch_bwd_tc_t<16>(P, L, maps, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace msl
