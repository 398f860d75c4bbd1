// Deformable slide attention: the CUDA-core ("gather") forward and backward kernels (sm_100a), one
// warp per (sample, query, head); the per-query bodies and their lane layout are in dsa_simt.cuh.
//
// Reference semantics (infinity/video/attention.py): grid construction :113-127 and :194-238,
// trilinear border sampling :240-273, scores / softmax / dropout / value sum :147-186, extra keys
// :159-173.

#include <math.h>

#include "dsa_attn.cuh"
#include "dsa_simt.cuh"
#include "msl_common.cuh"

namespace msl {

namespace {

__device__ __forceinline__ bool decode_item(const AttnParams& P, QueryPos& q) {
  const long long item = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long nitems = static_cast<long long>(P.B) * P.nh * P.Nq;
  if (item >= nitems) return false;
  q.r = item % P.Nq;
  const long long bh = item / P.Nq;
  q.head = static_cast<int>(bh % P.nh);
  q.b = static_cast<int>(bh / P.nh);
  const int tl = static_cast<int>(q.r / P.HW);
  const int rem = static_cast<int>(q.r - static_cast<long long>(tl) * P.HW);
  q.h = rem / P.W;
  q.w = rem - q.h * P.W;
  q.tg = P.q_frame0 + tl;
  return true;
}

}  // namespace

template <typename T, int VEC, int MAXC>
__global__ void __launch_bounds__(256) dsa_fwd_kernel(const AttnParams P) {
  QueryPos qp;
  if (!decode_item(P, qp)) return;
  fwd_query<T, VEC, MAXC>(P, qp);
}

template <typename T, int VEC, int MAXC>
__global__ void __launch_bounds__(256) dsa_bwd_kernel(const AttnParams P) {
  QueryPos qp;
  if (!decode_item(P, qp)) return;
  bwd_query<T, VEC, MAXC>(P, qp);
}

// dek[b, g, head*d + i] = sum_r extra_ds[b, head, r, g] * q[b, r, head*d + i]
// dev[b, g, head*d + i] = sum_r extra_p [b, head, r, g] * dout[b, r, head*d + i]
// grid: x over (g, i) pairs, y over (b, head), z over row chunks; float32 atomics into the outputs.
template <typename T>
__global__ void __launch_bounds__(256) dsa_extra_grad_kernel(const AttnParams P, int rows_per_chunk) {
  const int gi = blockIdx.x * blockDim.x + threadIdx.x;
  if (gi >= P.G * P.d) return;
  const int g = gi / P.d, i = gi - (gi / P.d) * P.d;
  const int head = blockIdx.y % P.nh, b = blockIdx.y / P.nh;
  const long long r0 = static_cast<long long>(blockIdx.z) * rows_per_chunk;
  const long long r1 = min(P.Nq, r0 + rows_per_chunk);
  const T* q = static_cast<const T*>(P.q) + static_cast<long long>(b) * P.Nq * P.q_ld + head * P.d + i;
  const T* dout = static_cast<const T*>(P.dout) + static_cast<long long>(b) * P.Nq * P.dout_ld + head * P.d + i;
  const float* ds = P.extra_ds + (static_cast<long long>(b) * P.nh + head) * P.Nq * P.G + g;
  const float* pp = P.extra_p + (static_cast<long long>(b) * P.nh + head) * P.Nq * P.G + g;
  float ak = 0.f, av = 0.f;
  for (long long r = r0; r < r1; ++r) {
    ak = fmaf(ds[r * P.G], to_f32<T>(q[r * P.q_ld]), ak);
    av = fmaf(pp[r * P.G], to_f32<T>(dout[r * P.dout_ld]), av);
  }
  const long long o = (static_cast<long long>(b) * P.G + g) * (static_cast<long long>(P.nh) * P.d) + head * P.d + i;
  atomicAdd(P.dek + o, ak);
  atomicAdd(P.dev + o, av);
}

// ------------------------------------------------------------------------------ dispatch
template <typename T, int VEC>
static cudaError_t launch_fwd_vec(const AttnParams& P, int maxc, cudaStream_t s) {
  const long long items = static_cast<long long>(P.B) * P.nh * P.Nq;
  const dim3 grid(static_cast<unsigned>((items + 7) / 8)), block(256);
  // bf16 16-byte chunks stop at 4 chunks per slot (head_dim 128); attn_chunking never asks for more
  constexpr int kLim = (VEC == 8) ? 4 : 8;
  switch (maxc) {
#define MSL_CASE(MC)                                            \
  case MC:                                                      \
    if constexpr (MC <= kLim) {                                 \
      dsa_fwd_kernel<T, VEC, MC><<<grid, block, 0, s>>>(P);         \
    } else {                                                    \
      return cudaErrorInvalidValue;                             \
    }                                                           \
    break;
    MSL_CASE(1) MSL_CASE(2) MSL_CASE(3) MSL_CASE(4)
    MSL_CASE(5) MSL_CASE(6) MSL_CASE(7) MSL_CASE(8)
#undef MSL_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T, int VEC>
static cudaError_t launch_bwd_vec(const AttnParams& P, int maxc, cudaStream_t s) {
  const long long items = static_cast<long long>(P.B) * P.nh * P.Nq;
  const dim3 grid(static_cast<unsigned>((items + 7) / 8)), block(256);
  // bf16 16-byte chunks stop at 4 chunks per slot (head_dim 128); attn_chunking never asks for more
  constexpr int kLim = (VEC == 8) ? 4 : 8;
  switch (maxc) {
#define MSL_CASE(MC)                                            \
  case MC:                                                      \
    if constexpr (MC <= kLim) {                                 \
      dsa_bwd_kernel<T, VEC, MC><<<grid, block, 0, s>>>(P);         \
    } else {                                                    \
      return cudaErrorInvalidValue;                             \
    }                                                           \
    break;
    MSL_CASE(1) MSL_CASE(2) MSL_CASE(3) MSL_CASE(4)
    MSL_CASE(5) MSL_CASE(6) MSL_CASE(7) MSL_CASE(8)
#undef MSL_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Chunking of the head dimension: VEC elements per 16-byte chunk when d allows, else 1.
// Returns false if the head dimension is not supported.
bool attn_chunking(int dtype, int d, int* vec, int* maxc) {
  const int v = (dtype == MSL_DTYPE_BF16) ? 8 : 4;
  if (d % v == 0) {
    const int mc = (d / v + 3) / 4;
    const int lim = (dtype == MSL_DTYPE_BF16) ? 4 : 8;
    if (mc > lim) return false;
    *vec = v;
    *maxc = mc;
    return true;
  }
  const int mc = (d + 3) / 4;
  if (mc > 8) return false;
  *vec = 1;
  *maxc = mc;
  return true;
}

cudaError_t launch_attn_fwd(const AttnParams& P, int vec, int maxc, cudaStream_t s) {
  if (P.dtype == MSL_DTYPE_BF16)
    return vec == 8 ? launch_fwd_vec<__nv_bfloat16, 8>(P, maxc, s) : launch_fwd_vec<__nv_bfloat16, 1>(P, maxc, s);
  return vec == 4 ? launch_fwd_vec<float, 4>(P, maxc, s) : launch_fwd_vec<float, 1>(P, maxc, s);
}

cudaError_t launch_attn_bwd(const AttnParams& P, int vec, int maxc, cudaStream_t s) {
  if (P.dtype == MSL_DTYPE_BF16)
    return vec == 8 ? launch_bwd_vec<__nv_bfloat16, 8>(P, maxc, s) : launch_bwd_vec<__nv_bfloat16, 1>(P, maxc, s);
  return vec == 4 ? launch_bwd_vec<float, 4>(P, maxc, s) : launch_bwd_vec<float, 1>(P, maxc, s);
}

cudaError_t launch_attn_extra_grad(const AttnParams& P, cudaStream_t s) {
  const int rows_per_chunk = 512;
  const dim3 grid(static_cast<unsigned>((P.G * P.d + 255) / 256), static_cast<unsigned>(P.B * P.nh),
                  static_cast<unsigned>((P.Nq + rows_per_chunk - 1) / rows_per_chunk));
  if (P.dtype == MSL_DTYPE_BF16)
    dsa_extra_grad_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(P, rows_per_chunk);
  else
    dsa_extra_grad_kernel<float><<<grid, 256, 0, s>>>(P, rows_per_chunk);
  return cudaGetLastError();
}

}  // namespace msl
