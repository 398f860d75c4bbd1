// Internal launch interface of the deformable-attention kernels.
#pragma once

#include <cuda.h>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace msl {

// Flattened, validated arguments of one attention call (host fills, kernels read by value).
struct AttnParams {
  int B, T, H, W, nh, d, kt, kh, kw, K, G;
  int q_frame0, q_frames, kv_frame0, kv_frames;
  int HW;
  long long Nq, Nkv;  // rows per sample
  int dtype;
  float scale;        // softmax scale
  float scale_log2;   // softmax scale * log2(e)
  float oscale;       // offset scale
  uint32_t drop_thresh;  // 0 = no dropout, else keep iff rng >= thresh (thresh = p * 2^32)
  float drop_keep_scale; // 1 / (1 - p)
  uint64_t seed;
  // operands (element strides)
  const void* q;  long long q_ld;
  const void* k;  long long k_ld;
  const void* v;  long long v_ld;
  const float* offsets; long long off_ld;
  const void* ek; const void* ev; long long e_ld;
  void* out; long long out_ld;        // forward: written; backward: read
  float* lse;
  float* probs;       // [B, nh, Nq, K] softmax weights before dropout (optional; tensor-core paths)
  void* saved;        // tensor-core forward -> backward: per-sample records + tile envelopes (optional)
  const float* off_bias;  // [nh*K*3] added to every offsets row (optional)
  const void* dout; long long dout_ld;
  void* dq; long long dq_ld;
  float* dk_acc; float* dv_acc; long long acc_ld;
  void* doffsets; long long doff_ld;
  int doff_bf16;      // doffsets element type: 0 float32, 1 bf16 (rounded to nearest even)
  float* extra_ds; float* extra_p;   // [B, nh, Nq, G] scratch
  float* dek; float* dev;            // [B, G, nh*d]
  uint32_t* status;
};

// the three offsets (channels 0, 1, 2) of window sample j of the offsets row `row` of head `head`, with
// the optional per-column bias added in one float32 rounding (as the materialised offsets + bias)
__device__ __forceinline__ void load_off3(const AttnParams& P, const float* row, int head, int j, float& o0, float& o1,
                                          float& o2) {
  o0 = row[3 * j];
  o1 = row[3 * j + 1];
  o2 = row[3 * j + 2];
  if (P.off_bias) {
    const float* b = P.off_bias + (static_cast<long long>(head) * P.K + j) * 3;
    o0 = __fadd_rn(o0, __ldg(b));
    o1 = __fadd_rn(o1, __ldg(b + 1));
    o2 = __fadd_rn(o2, __ldg(b + 2));
  }
}

// element i of the offset gradients in their element type
__device__ __forceinline__ void store_doff(const AttnParams& P, long long i, float v) {
  if (P.doff_bf16)
    static_cast<__nv_bfloat16*>(P.doffsets)[i] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(P.doffsets)[i] = v;
}

// Launch plan of the tensor-core kernels (key-envelope chunk capacity and shared-memory layout).
struct TcLaunch {
  int maxkeys;  // keys per envelope chunk (multiple of 16)
  int tma;      // K / V chunks by TMA tensor copies (set at launch when the tensor maps could be made)
  int rs;       // shared-memory row stride of a key (bf16 elements)
  int sld;      // row stride of the score / P~ buffer (floats)
  int tiles_h, tiles_w;
  long long tiles;
  size_t smem;
};
// Layout of `saved` (msl_dsa_saved_bytes): the forward's records [B, nh, Nq, K] uint64, then from
// saved_env_offset(P) on, per 4 x 8 query tile in CTA order, its raw envelope (8 int32: zlo, zhi, ylo,
// yhi, xlo, xhi, 0, 0).
__host__ __device__ inline long long saved_env_offset(const AttnParams& P) {
  return ((static_cast<long long>(P.B) * P.nh * P.Nq * P.K * 8) + 255) & ~255LL;
}
long long saved_bytes(const AttnParams& P);
bool tc_supported(const AttnParams& P);
bool tc_plan(const AttnParams& P, TcLaunch& L, int smem_limit);
cudaError_t launch_attn_fwd_tc(const AttnParams& P, const TcLaunch& L, cudaStream_t s);
bool tc_bwd_supported(const AttnParams& P);
bool tc_bwd_plan(const AttnParams& P, TcLaunch& L, int smem_limit);
cudaError_t launch_attn_bwd_tc(const AttnParams& P, const TcLaunch& L, cudaStream_t s);

bool attn_chunking(int dtype, int d, int* vec, int* maxc);
cudaError_t launch_attn_fwd(const AttnParams& P, int vec, int maxc, cudaStream_t s);
cudaError_t launch_attn_bwd(const AttnParams& P, int vec, int maxc, cudaStream_t s);
cudaError_t launch_attn_extra_grad(const AttnParams& P, cudaStream_t s);

// Depthwise 3D convolution (channels-last).
struct ConvParams {
  int B, T, H, W, C, kt, kh, kw;
  int in_frame0, in_frames, out_frame0, out_frames;
  int dtype;
  int HW;
};
// x has dtype P.dtype; aux and y have y_dtype.
cudaError_t launch_dwconv_fwd(const ConvParams& P, const void* x, long long x_ld, const float* wt,
                              const float* bias, const float* bias2, int epi, const void* aux,
                              long long aux_ld, void* y, long long y_ld, int y_dtype, bool flip,
                              cudaStream_t s);
// x has dtype P.dtype; dy has dy_dtype.
cudaError_t launch_dwconv_wgrad(const ConvParams& P, const void* dy, long long dy_ld, int dy_dtype,
                                const void* x, long long x_ld, float* dw, float* db, cudaStream_t s);

// Shared-memory tiled variants (dwconv_tiled.cu); cudaErrorNotSupported when the kernel width,
// channel count, alignment or shared-memory plan is outside what they cover (nothing is launched).
cudaError_t launch_dwconv_fwd_tiled(const ConvParams& P, const void* x, long long x_ld, const float* wt,
                                    const float* bias, const float* bias2, int epi, const void* aux, long long aux_ld,
                                    void* y, long long y_ld, int y_dtype, bool flip, cudaStream_t s);
cudaError_t launch_dwconv_wgrad_tiled(const ConvParams& P, const void* dy, long long dy_ld, int dy_dtype, const void* x,
                                      long long x_ld, float* dw, float* db, cudaStream_t s);

cudaError_t launch_offsets_absmax(const float* off, long long rows, long long ld, const float* bias, int heads, int taps,
                                  float oscale, float* out3, cudaStream_t s);
cudaError_t launch_convert_f32(const float* src, long long src_ld, void* dst, long long dst_ld,
                               int dtype, long long rows, long long cols, cudaStream_t s);

}  // namespace msl
