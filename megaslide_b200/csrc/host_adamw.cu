// Host-side optimizer kernels of the CPU-master trainer (megaslide_b200/stream.py): one-pass AdamW
// over a block's flat float32 master buffers and the gradient accumulation from the pinned slabs.
// Plain host code (OpenMP over the cores); replaces torch.optim.AdamW and the per-parameter
// gradient accumulation of the reference's CPU-master trainer (infinity/video/trainer.py:66-72,
// 176-221, 575-599), whose update runs as several full passes over the parameters.

#include <math.h>
#include <stdint.h>
#include <string.h>

#include "megaslide_b200.h"

namespace {

inline float bf16_to_f32(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// round to nearest even (NaN stays a quiet NaN)
inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return static_cast<uint16_t>((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

}  // namespace

extern "C" {

int msl_host_accumulate(float* dst, const void* src, int32_t src_dtype, int64_t n, int32_t overwrite,
                        double* sumsq) {
  if (!dst || !src || n < 0) return MSL_ERR_INVALID;
  if (src_dtype != MSL_DTYPE_F32 && src_dtype != MSL_DTYPE_BF16) return MSL_ERR_INVALID;
  double acc = 0.0;
  if (src_dtype == MSL_DTYPE_BF16) {
    const uint16_t* s = static_cast<const uint16_t*>(src);
#pragma omp parallel for reduction(+ : acc) schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      const float v = overwrite ? bf16_to_f32(s[i]) : dst[i] + bf16_to_f32(s[i]);
      dst[i] = v;
      acc += static_cast<double>(v) * v;
    }
  } else {
    const float* s = static_cast<const float*>(src);
#pragma omp parallel for reduction(+ : acc) schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      const float v = overwrite ? s[i] : dst[i] + s[i];
      dst[i] = v;
      acc += static_cast<double>(v) * v;
    }
  }
  if (sumsq) *sumsq = acc;
  return MSL_OK;
}

int msl_host_adamw(float* p, float* m, float* v, const float* g, int64_t n, float lr, float beta1, float beta2,
                   float eps, float weight_decay, int64_t step, float grad_scale, void* stage,
                   int32_t stage_dtype) {
  if (!p || !m || !v || !g || n < 0 || step < 1) return MSL_ERR_INVALID;
  if (stage && stage_dtype != MSL_DTYPE_F32 && stage_dtype != MSL_DTYPE_BF16) return MSL_ERR_INVALID;
  // torch.optim.AdamW (single tensor): p *= 1 - lr*wd; m = lerp(m, g, 1-b1); v = b2 v + (1-b2) g^2;
  // p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
  const float decay = 1.0f - lr * weight_decay;
  const float w1 = 1.0f - beta1, w2 = 1.0f - beta2;
  const float bc1 = 1.0f - static_cast<float>(pow(static_cast<double>(beta1), static_cast<double>(step)));
  const float bc2s = sqrtf(1.0f - static_cast<float>(pow(static_cast<double>(beta2), static_cast<double>(step))));
  const float step_size = lr / bc1;
  uint16_t* sb = stage_dtype == MSL_DTYPE_BF16 ? static_cast<uint16_t*>(stage) : nullptr;
  float* sf = stage_dtype == MSL_DTYPE_F32 ? static_cast<float*>(stage) : nullptr;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float gi = g[i] * grad_scale;
    float pi = p[i] * decay;
    const float mi = m[i] + w1 * (gi - m[i]);
    const float vi = beta2 * v[i] + w2 * gi * gi;
    pi -= step_size * (mi / (sqrtf(vi) / bc2s + eps));
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (sb) sb[i] = f32_to_bf16(pi);
    if (sf) sf[i] = pi;
  }
  return MSL_OK;
}

}  // extern "C"
