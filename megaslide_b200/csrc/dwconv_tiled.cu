// Shared-memory tiled depthwise 3D convolution over channels-last tokens: forward (also the input
// gradient, as a correlation with the flipped kernel) and weight gradient.
//
// One CTA owns a tile of TH rows x 32 columns of the volume, one group of 32 four-byte channel words
// (64 bf16 or 32 float32 channels) and a chunk of consecutive frames.  Input frames are staged in a
// ring of kt + 1 shared-memory slices (tile + kh/2, kw/2 halo, zero outside the volume; frames
// outside the input window read as zero) with cp.async:
// while output frame t is computed from slices t - kt/2 .. t + kt/2, slice t + kt/2 + 1 is loaded, so
// every input frame is fetched once per chunk and the fetch overlaps the arithmetic.  A warp owns one
// tile row and SEG consecutive columns (16, or 8 when the ring fits only 4 tile rows); each lane one
// channel word; the kw taps of a kernel row slide over SEG + kw - 1 register-resident inputs
// (SEG * kw * channels FMAs per SEG + kw - 1 shared loads).
//
// Replaces nn.Conv3d(C, C, k, padding=k//2, groups=C) of dw_conv (infinity/video/attention.py:58-65,
// 102) and offset_net[0] (attention.py:70-72, 105), forward and autograd backward.

#include <math.h>

#include "dsa_attn.cuh"
#include "dsa_tc.cuh"
#include "msl_common.cuh"

namespace msl {
namespace dwt {

constexpr int kTW = 32;   // tile columns
constexpr int kSeg = 16;  // consecutive outputs per thread along w
// weight gradient: 16 warps per CTA whatever the tile height, so the (kernel row, segment) items of a
// CTA spread over enough warps to hide the shared-memory latencies (at most 4 tile rows fit the ring)
constexpr int kWgradThreads = 512;

struct Plan {
  int th;        // tile rows (2 warps per row)
  int fpc;       // output frames per CTA
  int chunks, tiles_h, tiles_w, groups;
  int sr, sc;    // slice rows / columns (tile + halo)
  int dy_words;  // weight gradient: dy elements of one staged tile (0 for the forward)
  size_t smem;
  long long ctas;
};

// a0 += w0 * x0, a1 += w1 * x1 as one packed two-lane float32 FMA (sm_100 fma.rn.f32x2): each lane
// rounds exactly like fmaf, and the pair costs one issue slot instead of two.
__device__ __forceinline__ void fma_x2(float& a0, float& a1, float w0, float w1, float x0, float x1) {
  asm("{\n\t.reg .b64 a, w, x;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 w, {%2, %3};\n\tmov.b64 x, {%4, %5};\n\t"
      "fma.rn.f32x2 a, w, x, a;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(w0), "f"(w1), "f"(x0), "f"(x1));
}

// acc[e] += w[e] * x[e] over CV channels (packed pairs when CV == 2)
template <int CV>
__device__ __forceinline__ void fma_cv(float (&acc)[CV], const float (&w)[CV], const float (&x)[CV]) {
  if constexpr (CV == 2) {
    fma_x2(acc[0], acc[1], w[0], w[1], x[0], x[1]);
  } else {
#pragma unroll
    for (int e = 0; e < CV; ++e) acc[e] = fmaf(w[e], x[e], acc[e]);
  }
}

__device__ __forceinline__ float gelu_erf(float u) { return 0.5f * u * (1.f + erff(u * 0.70710678118654752f)); }

__device__ __forceinline__ float gelu_erf_grad(float u) {
  const float cdf = 0.5f * (1.f + erff(u * 0.70710678118654752f));
  const float pdf = 0.39894228040143268f * expf(-0.5f * u * u);
  return fmaf(u, pdf, cdf);
}

// four-byte word -> CV channels
template <typename T>
struct Word;
template <>
struct Word<__nv_bfloat16> {
  static constexpr int CV = 2;
  static __device__ __forceinline__ void unpack(uint32_t w, float (&o)[2]) {
    o[0] = bf16_lo(w);
    o[1] = bf16_hi(w);
  }
};
template <>
struct Word<float> {
  static constexpr int CV = 1;
  static __device__ __forceinline__ void unpack(uint32_t w, float (&o)[1]) { o[0] = __uint_as_float(w); }
};

// CV channels of type TY at p
template <typename TY, int CV>
__device__ __forceinline__ void load_cv(const TY* p, float (&o)[CV]) {
#pragma unroll
  for (int e = 0; e < CV; ++e) o[e] = to_f32<TY>(p[e]);
}
template <typename TY, int CV>
__device__ __forceinline__ void store_cv(TY* p, const float (&v)[CV]) {
  if constexpr (CV == 2 && sizeof(TY) == 2) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  } else if constexpr (CV == 2 && sizeof(TY) == 4) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
#pragma unroll
    for (int e = 0; e < CV; ++e) p[e] = from_f32<TY>(v[e]);
  }
}

// Stages input frame ti (global index) of sample b: rows h0 - kh/2 .. + sr - 1, columns w0 - kw/2 ..
// + sc - 1, channel words [c0, c0 + 32 words) as [sr][sc][32] words; zero outside the volume.
template <typename T>
__device__ __forceinline__ void load_slice(const ConvParams& P, const Plan& L, const T* x, long long x_ld, uint32_t* dst,
                                           int b, int ti, int h0, int w0, int c0) {
  const int ph = P.kh / 2, pw = P.kw / 2;
  const T* xb = x + (static_cast<long long>(b) * P.in_frames + (ti - P.in_frame0)) * P.HW * x_ld + c0;
  const int nchunk = L.sr * L.sc * 8;
  for (int i = threadIdx.x; i < nchunk; i += blockDim.x) {
    const int pos = i >> 3, ch = i & 7;
    const int row = pos / L.sc, col = pos - (pos / L.sc) * L.sc;
    const int h = h0 - ph + row, w = w0 - pw + col;
    uint32_t* d = dst + pos * 32 + ch * 4;
    if (h >= 0 && h < P.H && w >= 0 && w < P.W)
      tc::cp_async16(tc::smem_u32(d),
                     reinterpret_cast<const char*>(xb + (static_cast<long long>(h) * P.W + w) * x_ld) + ch * 16);
    else
      *reinterpret_cast<uint4*>(d) = make_uint4(0u, 0u, 0u, 0u);
  }
}

struct CtaPos {
  int b, ta, tb, h0, w0, cg;
};

__device__ __forceinline__ CtaPos decode(const ConvParams& P, const Plan& L) {
  long long id = blockIdx.x;
  CtaPos c;
  c.cg = static_cast<int>(id % L.groups);
  id /= L.groups;
  const int tw = static_cast<int>(id % L.tiles_w);
  id /= L.tiles_w;
  const int th = static_cast<int>(id % L.tiles_h);
  id /= L.tiles_h;
  const int chunk = static_cast<int>(id % L.chunks);
  c.b = static_cast<int>(id / L.chunks);
  c.h0 = th * L.th;
  c.w0 = tw * kTW;
  c.ta = P.out_frame0 + chunk * L.fpc;
  c.tb = min(P.out_frame0 + P.out_frames, c.ta + L.fpc);
  return c;
}

// y[p] = epi(sum_taps w[tap] x[p + tap - pad] + bias) (FLIP: w[K-1-tap], the input gradient).
// A warp owns SEG consecutive columns of one tile row: SEG = 16 when the tile has 8 rows (16 warps),
// 8 when the ring only fits 4 rows (kernel height 7), so the CTA still has 16 warps to hide the
// shared-memory and weight load latencies.
template <typename T, typename TY, int KW, bool FLIP, int SEG>
__global__ void __launch_bounds__(512, 1) dwconv_fwd_tiled_kernel(const ConvParams P, const Plan L, const T* __restrict__ x,
                                                               long long x_ld, const float* __restrict__ wt,
                                                               const float* __restrict__ bias,
                                                               const float* __restrict__ bias2, int epi,
                                                               const TY* __restrict__ aux, long long aux_ld,
                                                               TY* __restrict__ y, long long y_ld) {
  constexpr int CV = Word<T>::CV;
  constexpr int NIN = SEG + KW - 1;
  constexpr int NSEG = kTW / SEG;
  extern __shared__ __align__(16) uint32_t ring[];
  const CtaPos cp = decode(P, L);
  const int pt = P.kt / 2;
  const int nslots = P.kt + 1;
  const int slice_words = L.sr * L.sc * 32;
  const int base = cp.ta - pt;
  const int c0w = cp.cg * 32;  // first channel word of the group
  const int c0 = c0w * CV;
  for (int ti = max(P.in_frame0, cp.ta - pt); ti <= min(P.in_frame0 + P.in_frames - 1, cp.ta + pt); ++ti)
    load_slice<T>(P, L, x, x_ld, ring + ((ti - base) % nslots) * slice_words, cp.b, ti, cp.h0, cp.w0, c0);
  tc::cp_async_wait_all();
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp / NSEG, seg = warp % NSEG;
  const int h = cp.h0 + r, ws = cp.w0 + seg * SEG;
  const bool active = h < P.H && ws < P.W;
  const int c = c0 + lane * CV;
  float bsum[CV], b2v[CV];
#pragma unroll
  for (int e = 0; e < CV; ++e) {
    bsum[e] = bias ? __ldg(bias + c + e) : 0.f;
    b2v[e] = bias2 ? __ldg(bias2 + c + e) : 0.f;
  }
  for (int t = cp.ta; t < cp.tb; ++t) {
    const int tn = t + pt + 1;
    if (t + 1 < cp.tb && tn >= P.in_frame0 && tn < P.in_frame0 + P.in_frames)
      load_slice<T>(P, L, x, x_ld, ring + ((tn - base) % nslots) * slice_words, cp.b, tn, cp.h0, cp.w0, c0);
    if (active) {
      const long long orow0 = (static_cast<long long>(cp.b) * P.out_frames + (t - P.out_frame0)) * P.HW +
                              static_cast<long long>(h) * P.W + ws;
      float acc[SEG][CV];
#pragma unroll
      for (int j = 0; j < SEG; ++j)
#pragma unroll
        for (int e = 0; e < CV; ++e) acc[j][e] = 0.f;
      if (epi == MSL_EPI_ACCUM) {  // start from the buffer's own terms (loads issued together, before the taps)
#pragma unroll
        for (int j = 0; j < SEG; ++j)
          if (ws + j < P.W) load_cv<TY, CV>(y + (orow0 + j) * y_ld + c, acc[j]);
      }
      // GELU_GRAD (the non-transposed instantiations only: registers): the aux rows, loaded together before
      // the taps
      float avs[FLIP ? 1 : SEG][CV];
      if constexpr (!FLIP) {
        if (epi == MSL_EPI_GELU_GRAD) {
#pragma unroll
          for (int j = 0; j < SEG; ++j)
            if (ws + j < P.W) load_cv<TY, CV>(aux + (orow0 + j) * aux_ld + c, avs[j]);
        }
      }
      for (int it = 0; it < P.kt; ++it) {
        const int ti = t + it - pt;
        if (ti < P.in_frame0 || ti >= P.in_frame0 + P.in_frames) continue;  // zero outside the input frames
        const int itw = FLIP ? P.kt - 1 - it : it;
        const uint32_t* sl = ring + ((ti - base) % nslots) * slice_words;
        // weights of kernel row ih (flipped for the input gradient)
        auto load_w = [&](int ih, float (&dst)[KW][CV]) {
          const int ihw = FLIP ? P.kh - 1 - ih : ih;
          const float* wrow = wt + static_cast<long long>((itw * P.kh + ihw) * KW) * P.C + c;
#pragma unroll
          for (int iw = 0; iw < KW; ++iw) {
            const float* wp = wrow + static_cast<long long>(FLIP ? KW - 1 - iw : iw) * P.C;
            if constexpr (CV == 2) {
              const float2 v = __ldg(reinterpret_cast<const float2*>(wp));
              dst[iw][0] = v.x;
              dst[iw][CV - 1] = v.y;
            } else {
              dst[iw][0] = __ldg(wp);
            }
          }
        };
        float wv[KW][CV];
        load_w(0, wv);
        for (int ih = 0; ih < P.kh; ++ih) {
          const uint32_t* rowp = sl + ((r + ih) * L.sc + seg * SEG) * 32 + lane;
          float xin[NIN][CV];
#pragma unroll
          for (int j = 0; j < NIN; ++j) Word<T>::unpack(rowp[j * 32], xin[j]);
          // the next row's weights load while this row's FMAs run (the last row reloads itself)
          float wn[KW][CV];
          load_w(min(ih + 1, P.kh - 1), wn);
#pragma unroll
          for (int iw = 0; iw < KW; ++iw)
#pragma unroll
            for (int j = 0; j < SEG; ++j) fma_cv<CV>(acc[j], wv[iw], xin[j + iw]);
#pragma unroll
          for (int iw = 0; iw < KW; ++iw)
#pragma unroll
            for (int e = 0; e < CV; ++e) wv[iw][e] = wn[iw][e];
        }
      }
#pragma unroll
      for (int j = 0; j < SEG; ++j) {
        if (ws + j >= P.W) break;
        const long long orow = orow0 + j;
        float av[CV];
        if (epi == MSL_EPI_GELU_GRAD) {
          if constexpr (FLIP) {
            load_cv<TY, CV>(aux + orow * aux_ld + c, av);
          } else {
#pragma unroll
            for (int e = 0; e < CV; ++e) av[e] = avs[j][e];
          }
        }
        float out[CV];
#pragma unroll
        for (int e = 0; e < CV; ++e) {
          float u = acc[j][e] + bsum[e];
          if (epi == MSL_EPI_GELU)
            u = gelu_erf(u);
          else if (epi == MSL_EPI_GELU_GRAD)
            u = av[e] * gelu_erf_grad(u);
          else
            u += b2v[e];
          out[e] = u;
        }
        store_cv<TY, CV>(y + orow * y_ld + c, out);
      }
    }
    tc::cp_async_wait_all();
    __syncthreads();
  }
}

// CV consecutive dy values of one lane from shared memory (one 4- or 8-byte load for a channel pair)
template <typename TDY, int CV>
__device__ __forceinline__ void load_dy(const TDY* p, float (&g)[CV]) {
  if constexpr (CV == 2 && sizeof(TDY) == 2) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
    g[0] = bf16_lo(w);
    g[1] = bf16_hi(w);
  } else if constexpr (CV == 2 && sizeof(TDY) == 4) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    g[0] = v.x;
    g[1] = v.y;
  } else {
#pragma unroll
    for (int e = 0; e < CV; ++e) g[e] = to_f32<TDY>(p[e]);
  }
}

// Weight gradient: dw[tap][c] += sum_p dy[p][c] x[p + tap - pad][c], db[c] += sum_p dy[p][c].
// Items = (kernel row (it, ih) or the bias, 16-column segment); warp w owns items w, w + nwarps, ...
// for the whole CTA, accumulates them in registers over the chunk's frames and tile rows, and adds
// them to dw / db with one atomic per channel and tap at the end.
template <typename T, typename TDY, int KW, int MAXI>
__global__ void __launch_bounds__(kWgradThreads, 1) dwconv_wgrad_tiled_kernel(const ConvParams P, const Plan L,
                                                                 const TDY* __restrict__ dy, long long dy_ld,
                                                                 const T* __restrict__ x, long long x_ld,
                                                                 float* __restrict__ dw, float* __restrict__ db) {
  constexpr int CV = Word<T>::CV;
  constexpr int NIN = kSeg + KW - 1;
  extern __shared__ __align__(16) uint32_t ring[];
  const CtaPos cp = decode(P, L);
  const int pt = P.kt / 2;
  const int nslots = P.kt + 1;
  const int slice_words = L.sr * L.sc * 32;
  // dy tiles in their own type, double buffered: [2][th][32 cols][32 lanes][CV]
  TDY* dys = reinterpret_cast<TDY*>(ring + nslots * slice_words);
  const int base = cp.ta - pt;
  const int c0 = cp.cg * 32 * CV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int c = c0 + lane * CV;
  const int npairs = P.kt * P.kh;
  const int nitems = (npairs + (db ? 1 : 0)) * 2;

  // dy tile of frame t (rows h0.., columns w0..w0+31, this group's channels) with cp.async, zero
  // outside the volume; 16-byte chunks (rows are 16-byte aligned, host-checked)
  auto stage_dy = [&](int t, TDY* dst) {
    constexpr int kChunks = 32 * CV * static_cast<int>(sizeof(TDY)) / 16;  // per position
    const int n = L.th * kTW * kChunks;
    const TDY* base_dy = dy + (static_cast<long long>(cp.b) * P.out_frames + (t - P.out_frame0)) * P.HW * dy_ld + c0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int pos = i / kChunks, ch = i - (i / kChunks) * kChunks;
      const int row = pos / kTW, col = pos - (pos / kTW) * kTW;
      const int hh = cp.h0 + row, ww = cp.w0 + col;
      char* d = reinterpret_cast<char*>(dst + static_cast<size_t>(pos) * 32 * CV) + ch * 16;
      if (hh < P.H && ww < P.W)
        tc::cp_async16(tc::smem_u32(d),
                       reinterpret_cast<const char*>(base_dy + (static_cast<long long>(hh) * P.W + ww) * dy_ld) + ch * 16);
      else
        *reinterpret_cast<uint4*>(d) = make_uint4(0u, 0u, 0u, 0u);
    }
  };

  for (int ti = max(P.in_frame0, cp.ta - pt); ti <= min(P.in_frame0 + P.in_frames - 1, cp.ta + pt); ++ti)
    load_slice<T>(P, L, x, x_ld, ring + ((ti - base) % nslots) * slice_words, cp.b, ti, cp.h0, cp.w0, c0);
  stage_dy(cp.ta, dys);
  tc::cp_async_wait_all();
  __syncthreads();

  float acc[MAXI][KW][CV];
#pragma unroll
  for (int s = 0; s < MAXI; ++s)
#pragma unroll
    for (int iw = 0; iw < KW; ++iw)
#pragma unroll
      for (int e = 0; e < CV; ++e) acc[s][iw][e] = 0.f;

  int buf = 0;
  for (int t = cp.ta; t < cp.tb; ++t) {
    const int tn = t + pt + 1;
    if (t + 1 < cp.tb && tn >= P.in_frame0 && tn < P.in_frame0 + P.in_frames)
      load_slice<T>(P, L, x, x_ld, ring + ((tn - base) % nslots) * slice_words, cp.b, tn, cp.h0, cp.w0, c0);
    if (t + 1 < cp.tb) stage_dy(t + 1, dys + static_cast<size_t>(buf ^ 1) * L.dy_words);
    const TDY* dyt = dys + static_cast<size_t>(buf) * L.dy_words;
#pragma unroll
    for (int s = 0; s < MAXI; ++s) {
      const int item = warp + s * nwarps;
      if (item >= nitems) break;
      const int pair = item >> 1, seg = item & 1;
      if (cp.w0 + seg * kSeg >= P.W) continue;
      if (pair == npairs) {  // bias: sum of dy
        for (int r = 0; r < L.th; ++r) {
          const TDY* dp = dyt + (static_cast<size_t>(r * kTW + seg * kSeg) * 32 + lane) * CV;
#pragma unroll
          for (int j = 0; j < kSeg; ++j)
#pragma unroll
            for (int e = 0; e < CV; ++e) acc[s][0][e] += to_f32<TDY>(dp[j * 32 * CV + e]);
        }
        continue;
      }
      const int it = pair / P.kh, ih = pair - (pair / P.kh) * P.kh;
      const int ti = t + it - pt;
      if (ti < P.in_frame0 || ti >= P.in_frame0 + P.in_frames) continue;
      const uint32_t* sl = ring + ((ti - base) % nslots) * slice_words;
      for (int r = 0; r < L.th; ++r) {
        const uint32_t* rowp = sl + ((r + ih) * L.sc + seg * kSeg) * 32 + lane;
        const TDY* dp = dyt + (static_cast<size_t>(r * kTW + seg * kSeg) * 32 + lane) * CV;
        float xin[NIN][CV];
#pragma unroll
        for (int j = 0; j < NIN; ++j) Word<T>::unpack(rowp[j * 32], xin[j]);
#pragma unroll
        for (int j = 0; j < kSeg; ++j) {
          float g[CV];
          load_dy<TDY, CV>(dp + j * 32 * CV, g);
#pragma unroll
          for (int iw = 0; iw < KW; ++iw) fma_cv<CV>(acc[s][iw], g, xin[j + iw]);
        }
      }
    }
    tc::cp_async_wait_all();
    __syncthreads();
    buf ^= 1;
  }
#pragma unroll
  for (int s = 0; s < MAXI; ++s) {
    const int item = warp + s * nwarps;
    if (item >= nitems) break;
    const int pair = item >> 1;
    if (pair == npairs) {
#pragma unroll
      for (int e = 0; e < CV; ++e) atomicAdd(db + c + e, acc[s][0][e]);
      continue;
    }
    float* drow = dw + static_cast<long long>(pair * KW) * P.C + c;
#pragma unroll
    for (int iw = 0; iw < KW; ++iw)
#pragma unroll
      for (int e = 0; e < CV; ++e) atomicAdd(drow + static_cast<long long>(iw) * P.C + e, acc[s][iw][e]);
  }
}

// ------------------------------------------------------------------------------ host side
int smem_limit() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
  return v - 1024;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Tile rows, frame chunking and shared memory of a launch; false when the tiled kernels do not apply.
bool make_plan(const ConvParams& P, int cv, int dy_cv_bytes, int max_threads, Plan& L) {
  const int kw = P.kw;
  if (kw != 1 && kw != 3 && kw != 5 && kw != 7) return false;
  if (P.C % (32 * cv) != 0) return false;
  const int limit = smem_limit();
  L.sc = kTW + kw - 1;
  L.th = 0;
  for (int th = max_threads / 64; th >= 1; th >>= 1) {
    if (th > 1 && th / 2 >= P.H) continue;  // no taller than the volume needs
    const int sr = th + P.kh - 1;
    const size_t ring = static_cast<size_t>(P.kt + 1) * sr * L.sc * 32 * 4;
    const size_t dyb = dy_cv_bytes ? static_cast<size_t>(2) * th * kTW * 32 * dy_cv_bytes : 0;
    if (ring + dyb <= static_cast<size_t>(limit)) {
      L.th = th;
      L.sr = sr;
      L.smem = ring + dyb;
      L.dy_words = dy_cv_bytes ? th * kTW * 32 * cv : 0;  // elements of the dy type per buffer
      break;
    }
  }
  if (L.th == 0) return false;
  L.tiles_h = (P.H + L.th - 1) / L.th;
  L.tiles_w = (P.W + kTW - 1) / kTW;
  L.groups = P.C / (32 * cv);
  // frames per CTA: enough CTAs for ~8 waves of 148 SMs, at most 16 frames per chunk
  const long long per_frame = static_cast<long long>(P.B) * L.tiles_h * L.tiles_w * L.groups;
  long long want = (per_frame * P.out_frames + 148LL * 8 - 1) / (148LL * 8);
  L.fpc = static_cast<int>(want < 1 ? 1 : (want > 16 ? 16 : want));
  if (L.fpc > P.out_frames) L.fpc = P.out_frames;
  L.chunks = (P.out_frames + L.fpc - 1) / L.fpc;
  L.ctas = per_frame * L.chunks;
  return L.ctas <= 0x7fffffffLL;
}

template <typename T, typename TY, int KW, bool FLIP, int SEG>
cudaError_t fwd_launch(const ConvParams& P, const Plan& L, const void* x, long long x_ld, const float* wt,
                       const float* bias, const float* bias2, int epi, const void* aux, long long aux_ld, void* y,
                       long long y_ld, cudaStream_t s) {
  auto k = dwconv_fwd_tiled_kernel<T, TY, KW, FLIP, SEG>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  k<<<static_cast<unsigned>(L.ctas), L.th * (kTW / SEG) * 32, L.smem, s>>>(P, L, static_cast<const T*>(x), x_ld, wt, bias, bias2, epi,
                                                            static_cast<const TY*>(aux), aux_ld, static_cast<TY*>(y),
                                                            y_ld);
  return cudaGetLastError();
}

template <typename T, typename TY, bool FLIP, int SEG>
cudaError_t fwd_kw(const ConvParams& P, const Plan& L, const void* x, long long x_ld, const float* wt, const float* bias,
                   const float* bias2, int epi, const void* aux, long long aux_ld, void* y, long long y_ld,
                   cudaStream_t s) {
  switch (P.kw) {
    case 1: return fwd_launch<T, TY, 1, FLIP, SEG>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
    case 3: return fwd_launch<T, TY, 3, FLIP, SEG>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
    case 5: return fwd_launch<T, TY, 5, FLIP, SEG>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
    default: return fwd_launch<T, TY, 7, FLIP, SEG>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
  }
}

// 8-column segments when the plan has 4 tile rows (16 warps instead of 8), else 16-column ones
template <typename T, typename TY, bool FLIP>
cudaError_t fwd_seg(const ConvParams& P, const Plan& L, const void* x, long long x_ld, const float* wt,
                    const float* bias, const float* bias2, int epi, const void* aux, long long aux_ld, void* y,
                    long long y_ld, cudaStream_t s) {
  if (L.th == 4) return fwd_kw<T, TY, FLIP, 8>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
  return fwd_kw<T, TY, FLIP, kSeg>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
}

template <typename T, typename TY>
cudaError_t fwd_flip(const ConvParams& P, const Plan& L, bool flip, const void* x, long long x_ld, const float* wt,
                     const float* bias, const float* bias2, int epi, const void* aux, long long aux_ld, void* y,
                     long long y_ld, cudaStream_t s) {
  if (flip) return fwd_seg<T, TY, true>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
  return fwd_seg<T, TY, false>(P, L, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
}

template <typename T, typename TDY, int KW, int MAXI>
cudaError_t wgrad_launch(const ConvParams& P, const Plan& L, const void* dy, long long dy_ld, const void* x,
                         long long x_ld, float* dw, float* db, cudaStream_t s) {
  auto k = dwconv_wgrad_tiled_kernel<T, TDY, KW, MAXI>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  k<<<static_cast<unsigned>(L.ctas), kWgradThreads, L.smem, s>>>(P, L, static_cast<const TDY*>(dy), dy_ld,
                                                            static_cast<const T*>(x), x_ld, dw, db);
  return cudaGetLastError();
}

template <typename T, typename TDY, int MAXI>
cudaError_t wgrad_kw(const ConvParams& P, const Plan& L, const void* dy, long long dy_ld, const void* x, long long x_ld,
                     float* dw, float* db, cudaStream_t s) {
  switch (P.kw) {
    case 1: return wgrad_launch<T, TDY, 1, MAXI>(P, L, dy, dy_ld, x, x_ld, dw, db, s);
    case 3: return wgrad_launch<T, TDY, 3, MAXI>(P, L, dy, dy_ld, x, x_ld, dw, db, s);
    case 5: return wgrad_launch<T, TDY, 5, MAXI>(P, L, dy, dy_ld, x, x_ld, dw, db, s);
    default: return wgrad_launch<T, TDY, 7, MAXI>(P, L, dy, dy_ld, x, x_ld, dw, db, s);
  }
}

template <typename T, typename TDY>
cudaError_t wgrad_items(const ConvParams& P, const Plan& L, int maxi, const void* dy, long long dy_ld, const void* x,
                        long long x_ld, float* dw, float* db, cudaStream_t s) {
  if (maxi <= 2) return wgrad_kw<T, TDY, 2>(P, L, dy, dy_ld, x, x_ld, dw, db, s);
  if (maxi <= 4) return wgrad_kw<T, TDY, 4>(P, L, dy, dy_ld, x, x_ld, dw, db, s);
  return wgrad_kw<T, TDY, 6>(P, L, dy, dy_ld, x, x_ld, dw, db, s);
}

}  // namespace dwt

cudaError_t launch_dwconv_fwd_tiled(const ConvParams& P, const void* x, long long x_ld, const float* wt,
                                    const float* bias, const float* bias2, int epi, const void* aux, long long aux_ld,
                                    void* y, long long y_ld, int y_dtype, bool flip, cudaStream_t s) {
  const bool xb = P.dtype == MSL_DTYPE_BF16, yb = y_dtype == MSL_DTYPE_BF16;
  const int cv = xb ? 2 : 1;
  const size_t es = xb ? 2 : 4, ys = yb ? 2 : 4;
  if (!dwt::aligned(x, 16) || (x_ld * es) % 16 != 0) return cudaErrorNotSupported;
  if (!dwt::aligned(y, cv * ys) || y_ld % cv != 0 || !dwt::aligned(wt, 4 * cv)) return cudaErrorNotSupported;
  if (epi == MSL_EPI_GELU_GRAD && (!dwt::aligned(aux, cv * ys) || aux_ld % cv != 0)) return cudaErrorNotSupported;
  dwt::Plan L{};
  if (!dwt::make_plan(P, cv, 0, 512, L)) return cudaErrorNotSupported;
  if (xb) {
    if (yb) return dwt::fwd_flip<__nv_bfloat16, __nv_bfloat16>(P, L, flip, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
    return dwt::fwd_flip<__nv_bfloat16, float>(P, L, flip, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
  }
  if (yb) return dwt::fwd_flip<float, __nv_bfloat16>(P, L, flip, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
  return dwt::fwd_flip<float, float>(P, L, flip, x, x_ld, wt, bias, bias2, epi, aux, aux_ld, y, y_ld, s);
}

cudaError_t launch_dwconv_wgrad_tiled(const ConvParams& P, const void* dy, long long dy_ld, int dy_dtype, const void* x,
                                      long long x_ld, float* dw, float* db, cudaStream_t s) {
  const bool xb = P.dtype == MSL_DTYPE_BF16, yb = dy_dtype == MSL_DTYPE_BF16;
  const int cv = xb ? 2 : 1;
  const size_t es = xb ? 2 : 4, ys = yb ? 2 : 4;
  if (!dwt::aligned(x, 16) || (x_ld * es) % 16 != 0) return cudaErrorNotSupported;
  if (!dwt::aligned(dy, 16) || (dy_ld * ys) % 16 != 0) return cudaErrorNotSupported;
  dwt::Plan L{};
  if (!dwt::make_plan(P, cv, static_cast<int>(cv * ys), 256, L)) return cudaErrorNotSupported;
  const int nwarps = dwt::kWgradThreads / 32;
  const int nitems = (P.kt * P.kh + (db ? 1 : 0)) * 2;
  const int maxi = (nitems + nwarps - 1) / nwarps;
  if (maxi > 6) return cudaErrorNotSupported;
  if (xb) {
    if (yb) return dwt::wgrad_items<__nv_bfloat16, __nv_bfloat16>(P, L, maxi, dy, dy_ld, x, x_ld, dw, db, s);
    return dwt::wgrad_items<__nv_bfloat16, float>(P, L, maxi, dy, dy_ld, x, x_ld, dw, db, s);
  }
  if (yb) return dwt::wgrad_items<float, __nv_bfloat16>(P, L, maxi, dy, dy_ld, x, x_ld, dw, db, s);
  return dwt::wgrad_items<float, float>(P, L, maxi, dy, dy_ld, x, x_ld, dw, db, s);
}

}  // namespace msl
