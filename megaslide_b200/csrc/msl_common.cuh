// Shared device helpers for the megaslide_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "megaslide_b200.h"

namespace msl {

constexpr unsigned kFull = 0xffffffffu;
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- element access
// A "chunk" is VEC consecutive elements loaded as one 16-byte vector (VEC = 16/sizeof(T)) or,
// for head dims that are not a multiple of that, a single element (VEC = 1).

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <typename T, int VEC>
struct Chunk;

template <>
struct Chunk<float, 4> {
  static __device__ __forceinline__ void load(const float* p, float (&o)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&o)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
  }
};

template <>
struct Chunk<float, 1> {
  static __device__ __forceinline__ void load(const float* p, float (&o)[1]) { o[0] = __ldg(p); }
  static __device__ __forceinline__ void store(float* p, const float (&o)[1]) { p[0] = o[0]; }
};

template <>
struct Chunk<__nv_bfloat16, 8> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[8]) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    o[0] = bf16_lo(v.x); o[1] = bf16_hi(v.x); o[2] = bf16_lo(v.y); o[3] = bf16_hi(v.y);
    o[4] = bf16_lo(v.z); o[5] = bf16_hi(v.z); o[6] = bf16_lo(v.w); o[7] = bf16_hi(v.w);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&o)[8]) {
    uint4 v;
    __nv_bfloat162 t;
    t = __floats2bfloat162_rn(o[0], o[1]); v.x = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(o[2], o[3]); v.y = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(o[4], o[5]); v.z = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(o[6], o[7]); v.w = *reinterpret_cast<uint32_t*>(&t);
    *reinterpret_cast<uint4*>(p) = v;
  }
};

template <>
struct Chunk<__nv_bfloat16, 1> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[1]) {
    o[0] = __bfloat162float(p[0]);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&o)[1]) {
    p[0] = __float2bfloat16_rn(o[0]);
  }
};

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Accumulate VEC floats into a float32 row with global atomics (vector atomics when aligned).
template <int VEC>
__device__ __forceinline__ void atomic_add_chunk(float* p, const float (&v)[VEC]) {
  if constexpr (VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC; i += 4)
      atomicAdd(reinterpret_cast<float4*>(p + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) atomicAdd(p + i, v[i]);
  }
}

// ---------------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// ---------------------------------------------------------------- sampling coordinates
// The reference builds its grid in float32 (attention.py:209-236) with
//   base = 2*a / max(S-1, 1) - 1,   a = position + window index - k//2,
// adds offset/(S'-1) where the offset channel feeding grid axis x (W) is channel 0 divided by
// (T-1), channel 1 feeds y (H) divided by (H-1) and channel 2 feeds z (T) divided by (W-1)
// (attention.py:118-127 stacked as (w, h, t) at :236), then grid_sample(align_corners=False,
// padding_mode='border') unnormalises p = ((g + 1)*S - 1)/2 and clamps p to [0, S-1].
// Every step is one correctly rounded float32 operation in that order (the explicit _rn
// intrinsics keep the compiler from contracting them into FMAs), so the voxel coordinate and
// therefore the floor() corner choice is bit-identical to the reference's CPU float32 path.

__device__ __forceinline__ float base_grid(int a, int S) {
  const float den = static_cast<float>(S > 1 ? S - 1 : 1);
  return __fsub_rn(__fdiv_rn(static_cast<float>(2 * a), den), 1.0f);
}

// grid -> clamped pixel coordinate (border padding, align_corners=False).
__device__ __forceinline__ float unnormalize_clip(float g, int S) {
  const float v = __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(g, 1.0f), static_cast<float>(S)), 1.0f), 0.5f);
  const float hi = static_cast<float>(S - 1);
  // std::min(S-1, std::max(v, 0)) including its NaN behaviour (a NaN coordinate becomes S-1)
  const float lo = (v < 0.f) ? 0.f : v;
  return (lo < hi) ? lo : hi;
}

// d p / d grid after clamping: S/2 strictly inside (0, S-1), 0 on or beyond the border
// (grid_sampler's clip_coordinates_set_grad treats the border itself as outside).
__device__ __forceinline__ float clip_grad_mult(float p, int S) {
  return (p > 0.f && p < static_cast<float>(S - 1)) ? 0.5f * static_cast<float>(S) : 0.f;
}

struct SampleGeom {
  int T, H, W;       // global volume
  int kt, kh, kw;
  float oscale;
};

// Clamped voxel coordinates (pt, ph, pw) of window sample j of the query at global (t, h, w)
// from its three raw offsets o[0..2].
__device__ __forceinline__ void sample_coords(const SampleGeom& g, int t, int h, int w, int j,
                                              float o0, float o1, float o2, float& pt, float& ph,
                                              float& pw) {
  const int khw = g.kh * g.kw;
  const int it = j / khw;
  const int rem = j - it * khw;
  const int ih = rem / g.kw;
  const int iw = rem - ih * g.kw;
  float gx = base_grid(w + iw - g.kw / 2, g.W);
  float gy = base_grid(h + ih - g.kh / 2, g.H);
  float gz = base_grid(t + it - g.kt / 2, g.T);
  if (g.T > 1) gx = __fadd_rn(gx, __fdiv_rn(__fmul_rn(o0, g.oscale), static_cast<float>(g.T - 1)));
  if (g.H > 1) gy = __fadd_rn(gy, __fdiv_rn(__fmul_rn(o1, g.oscale), static_cast<float>(g.H - 1)));
  if (g.W > 1) gz = __fadd_rn(gz, __fdiv_rn(__fmul_rn(o2, g.oscale), static_cast<float>(g.W - 1)));
  pw = unnormalize_clip(gx, g.W);
  ph = unnormalize_clip(gy, g.H);
  pt = unnormalize_clip(gz, g.T);
}

// Trilinear weight factors along one axis in grid_sampler's form: the lower corner gets
// (i0 + 1) - p, the upper corner p - i0.
__device__ __forceinline__ float axis_weight(float p, int i0, int upper) {
  return upper ? __fsub_rn(p, static_cast<float>(i0)) : __fsub_rn(static_cast<float>(i0 + 1), p);
}

// ---------------------------------------------------------------- dropout
// Counter-based keep decision: SplitMix64 (Steele, Lea & Flood, OOPSLA 2014) finaliser applied to
// seed ^ (index * golden-ratio constant).  Index = global (unsharded) position of the softmax
// weight, so every sharding of the volume drops the same weights.
__device__ __host__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ __forceinline__ bool dropout_keep(uint64_t seed, uint64_t index, uint32_t threshold) {
  const uint64_t r = splitmix64(seed ^ (index * 0xD1B54A32D192ED03ull));
  return static_cast<uint32_t>(r >> 32) >= threshold;
}

}  // namespace msl
