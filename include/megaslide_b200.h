/*
 * megaslide_b200 — C ABI of the B200 (sm_100a) 3D Deformable Slide Attention kernels.
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream (passed as void*, a
 * cudaStream_t).  All device buffers are owned by the caller.  Entry points never allocate
 * device memory, never synchronise the stream and never abort: they return MSL_OK (0) or a
 * negative error code, and msl_last_error() then holds a one-line description (thread-local).
 * Work is stream-ordered on the caller's stream.
 *
 * Layout conventions (all row-major, "rows" are tokens, "ld" is the row stride in elements):
 *   tokens of one sample are ordered n = (t*H + h)*W + w, exactly like the reference's
 *   x[B, N, D] (infinity/video/attention.py:85-99);
 *   a C-channel token row holds heads back to back: channel = head*d + i.
 *   Raw offsets are float32 [B, rows, nh*kt*kh*kw*3] in the reference's 1x1-conv channel order
 *   ((((head*kt + it)*kh + ih)*kw + iw)*3 + axis)   (infinity/video/attention.py:105-111).
 *
 * Sharding along time: the geometry names the GLOBAL frame count T (coordinates are normalised
 * with it, as in the reference) plus the window of frames a call reads or writes, so one rank can
 * own query frames [q_frame0, q_frame0+q_frames) while its K/V buffers hold frames
 * [kv_frame0, kv_frame0+kv_frames) (its own frames plus halo).  Single-GPU callers set
 * q_frame0 = kv_frame0 = 0 and q_frames = kv_frames = T.
 */
#ifndef MEGASLIDE_B200_H
#define MEGASLIDE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MSL_ABI_VERSION 4  /* 2: msl_dsa_fwd_io / msl_dsa_bwd_io end with `saved`; 3: msl_dsa_bwd_io ends with
                              `doff_dtype`; 4: both end with `offset_bias`, msl_offsets_absmax takes a bias */

/* return codes */
#define MSL_OK 0
#define MSL_ERR_INVALID (-1)     /* bad argument (shape, pointer, stride, alignment) */
#define MSL_ERR_UNSUPPORTED (-2) /* valid but not implemented (e.g. head_dim too large) */
#define MSL_ERR_CUDA (-3)        /* a CUDA runtime call failed (launch error) */
#define MSL_ERR_WORKSPACE (-4)   /* workspace missing or too small */

/* element types of activations */
#define MSL_DTYPE_F32 0
#define MSL_DTYPE_BF16 1

/* bits of the optional device status word */
#define MSL_STATUS_HALO_MISS 1u  /* a sample corner fell in a frame the K/V buffers do not hold */
#define MSL_STATUS_TC_RANGE 2u   /* tensor-core path: a tile's key envelope exceeded what its sample
                                    records encode (a temporal span over 29 frames, or over 255 rows or
                                    columns: offsets of tens of voxels); the kernel computed that tile
                                    with the CUDA-core gather instead, forward and backward alike, so
                                    the results are valid (informational) */
#define MSL_STATUS_TIMEOUT 4u    /* tensor-core path: a CTA's TMA copies did not complete within a second;
                                    it stopped waiting, waited at most one more second for the copies it
                                    had issued, skipped every phase that reads the copied keys, and its
                                    results are not valid */

/* kernel family */
#define MSL_ALGO_AUTO 0 /* tensor-core envelope kernels when supported (bf16, head_dim % 8 == 0, <= 128) */
#define MSL_ALGO_SIMT 1 /* CUDA-core gather kernels (float32 and bf16, any head_dim <= 128) */
#define MSL_ALGO_TC 2   /* tensor-core envelope kernels; MSL_ERR_UNSUPPORTED when not applicable */

/* ----------------------------------------------------------------------------------------------
 * Geometry of one deformable-slide-attention call.
 * Replaces the shape logic of DeformableSlideAttention3D.forward / _get_base_grid
 * (infinity/video/attention.py:93-127, 194-238).
 * ---------------------------------------------------------------------------------------------- */
typedef struct msl_dsa_geometry {
  int32_t batch;      /* B */
  int32_t frames;     /* T of the GLOBAL volume */
  int32_t height;     /* H */
  int32_t width;      /* W */
  int32_t heads;      /* nh */
  int32_t head_dim;   /* d  (hidden = nh*d) */
  int32_t kt, kh, kw; /* neighbourhood (kernel_size) */
  int32_t extra;      /* G extra keys/values appended to every neighbourhood, 0 = none */
  int32_t q_frame0;   /* first global frame of the query rows of this call */
  int32_t q_frames;   /* number of query frames: rows per sample = q_frames*H*W */
  int32_t kv_frame0;  /* first global frame held by the K/V buffers */
  int32_t kv_frames;  /* number of frames held by the K/V buffers */
  int32_t dtype;      /* MSL_DTYPE_* of q, k, v, ek, ev, out, dout, dq, dk, dv */
  float softmax_scale; /* multiplies q.k (reference: 1/sqrt(d), attention.py:176) */
  float offset_scale;  /* multiplies the raw offsets (attention.py:106) */
  float dropout_p;     /* dropout on the softmax weights (attention.py:180); 0 = off */
  uint64_t dropout_seed;
  int32_t algo;        /* MSL_ALGO_* */
} msl_dsa_geometry;

/* Forward operands.  q: [B, q rows, >=nh*d]; k, v: [B, kv rows, >=nh*d];
 * ek, ev: [B, G, >=nh*d] already projected by k_proj / v_proj (attention.py:163-164), or NULL;
 * out: [B, q rows, >=nh*d] attention result before out_proj (attention.py:183-186);
 * lse: float32 [B, nh, q rows], base-2 log-sum-exp of the log2(e)-scaled scores (saved for
 * the backward pass); status: optional device word OR-ed with MSL_STATUS_* bits;
 * probs: optional float32 [B, nh, q rows, kt*kh*kw], the softmax weight of every window sample
 * before dropout (extra keys excluded), written only by the tensor-core path (MSL_ALGO_TC, or
 * MSL_ALGO_AUTO when it applies) and consumed by the tensor-core backward; NULL = not saved.
 * saved: optional msl_dsa_saved_bytes(geom) bytes (16-byte aligned): the tensor-core forward's
 * per-sample records (trilinear corner, fractions, interior and dropout flags) and per-tile key
 * envelopes, which the tensor-core backward reads instead of recomputing the sample coordinates
 * from the offsets; written only by the tensor-core path.  NULL = not saved.
 * offset_bias: optional float32 [nh*kt*kh*kw*3] added to every offsets row before use (the offset
 * predictor's 1x1-conv bias, attention.py:70-74: offsets[r, c] + offset_bias[c] in one float32
 * rounding, exactly the materialised sum); NULL = the offsets are used as they are. */
typedef struct msl_dsa_fwd_io {
  const void* q;   int64_t q_ld;
  const void* k;   int64_t k_ld;
  const void* v;   int64_t v_ld;
  const float* offsets; int64_t off_ld;
  const void* ek;  const void* ev; int64_t e_ld;
  void* out;       int64_t out_ld;
  float* lse;
  uint32_t* status;
  float* probs;
  void* saved;
  const float* offset_bias;
} msl_dsa_fwd_io;

/* Backward operands.  Inputs as in the forward plus out/lse from it and dout = dL/d out.
 * Outputs: dq [B, q rows, nh*d] (dtype, overwritten); doffsets [B, q rows, nh*K*3] of type doff_dtype
 * (MSL_DTYPE_F32, the zero default, or MSL_DTYPE_BF16: the float32 value rounded to nearest even;
 * overwritten, gradient w.r.t. the RAW offsets, offset_scale included); dek, dev float32
 * [B, G, nh*d] (overwritten; required when G > 0).
 * dK / dV, two modes:
 *   dk_acc == NULL: dk, dv [B, kv rows, nh*d] (dtype) are overwritten; float32 accumulators
 *                   live in the workspace.
 *   dk_acc != NULL: float32 dk_acc, dv_acc [B, kv rows, >=nh*d] (row stride acc_ld) are
 *                   ACCUMULATED into (not cleared), dk / dv are not touched.  Used by the
 *                   time-sharded path, which reduces halo rows across ranks before converting.
 * probs, saved: the tensor-core forward's optional outputs (see msl_dsa_fwd_io), from the forward of
 * the same operands; offset_bias as in msl_dsa_fwd_io (the same as the forward's).  When both are given (bf16, no extra keys) the tensor-core backward runs;
 * otherwise the CUDA-core backward. */
typedef struct msl_dsa_bwd_io {
  const void* q;   int64_t q_ld;
  const void* k;   int64_t k_ld;
  const void* v;   int64_t v_ld;
  const float* offsets; int64_t off_ld;
  const void* ek;  const void* ev; int64_t e_ld;
  const void* out; int64_t out_ld;
  const float* lse;
  const void* dout; int64_t dout_ld;
  void* dq;        int64_t dq_ld;
  void* dk;        void* dv;  int64_t dkv_ld;
  float* dk_acc;   float* dv_acc; int64_t acc_ld;
  void* doffsets;  int64_t doff_ld;
  float* dek;      float* dev;
  uint32_t* status;
  const float* probs;
  const void* saved;
  int32_t doff_dtype;
  const float* offset_bias;
} msl_dsa_bwd_io;

/* Size in bytes of the `saved` buffer of msl_dsa_fwd_io / msl_dsa_bwd_io for this geometry
 * (0 for an invalid geometry). */
size_t msl_dsa_saved_bytes(const msl_dsa_geometry* geom);

/* Forward of the deformable gather attention: for every query, head and window sample, the
 * trilinear border-clamped sample of K and V at the offset grid position (reference
 * grid_sample(bilinear, border, align_corners=False), attention.py:113-127, 240-273), softmax over
 * the kt*kh*kw samples (+G extra keys) and the weighted sum of the sampled values
 * (attention.py:147-186). */
int msl_dsa_attn_fwd(const msl_dsa_geometry* geom, const msl_dsa_fwd_io* io, void* stream);

/* Bytes of device workspace msl_dsa_attn_bwd needs.  accumulate_mode != 0: dk_acc is supplied
 * by the caller, so only the extra-key scratch is counted. */
size_t msl_dsa_attn_bwd_workspace_bytes(const msl_dsa_geometry* geom, int32_t accumulate_mode);

/* Backward of msl_dsa_attn_fwd: dQ, dK, dV, d(offsets), d(ek), d(ev).  Replaces autograd through
 * attention.py:113-186 (grid_sampler_3d_backward, bmm and softmax backward). */
int msl_dsa_attn_bwd(const msl_dsa_geometry* geom, const msl_dsa_bwd_io* io, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Capacity of the scratch array msl_dsa_attn_bwd_noalloc uses (64 MiB on every GPU that loads
 * the library, held until the process exits). */
#define MSL_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)

/* msl_dsa_attn_bwd without a caller-provided workspace: it allocates nothing.  No counterpart in
 * the reference.  For callers that cannot call cudaMalloc - a plugin whose host engine owns every
 * byte of device memory through its own pool, or code that must not trigger the implicit device
 * synchronisation and possible out-of-memory failure of an allocation in the middle of a step.
 * Its float32 scratch lives in one static device array of MSL_NOALLOC_SCRATCH_BYTES per GPU; a
 * problem needing more (msl_dsa_attn_bwd_workspace_bytes) is rejected with MSL_ERR_WORKSPACE.
 * The first call on a device looks the array's address up (call it once before any stream
 * capture); the address is kept for the life of the process, so the entry point must not be used
 * after cudaDeviceReset on that device (a new context places the array elsewhere).  Every call shares the array and clears what it accumulates into, so two calls whose
 * work overlaps on the GPU (different streams, or different threads) race and must be ordered by
 * the caller.  Arguments and results are those of msl_dsa_attn_bwd. */
int msl_dsa_attn_bwd_noalloc(const msl_dsa_geometry* geom, const msl_dsa_bwd_io* io, void* stream);

/* ----------------------------------------------------------------------------------------------
 * Depthwise 3D convolution over channels-last tokens [B, frames*H*W, C] with zero padding
 * (kt/2, kh/2, kw/2) at the borders of the GLOBAL volume.  Replaces nn.Conv3d(groups=C) of
 * dw_conv (attention.py:58-65, 102) and offset_net[0..1] (attention.py:70-72, 105).
 * weight: float32 [kt*kh*kw, C] (tap-major: reference weight[c,0,it,ih,iw] at row (it*kh+ih)*kw+iw).
 * ---------------------------------------------------------------------------------------------- */
typedef struct msl_dwconv_geometry {
  int32_t batch, frames, height, width, channels; /* frames = GLOBAL T */
  int32_t kt, kh, kw;
  int32_t in_frame0, in_frames;   /* frames held by the input buffer */
  int32_t out_frame0, out_frames; /* frames produced / reduced over */
  int32_t dtype;                  /* MSL_DTYPE_* of the activation buffers */
  int32_t zero_outside;           /* 0: the input frames must hold every tap of the output frames
                                     (frames outside the volume are zero padding); 1: frames outside
                                     the input window also read as zero -- the adjoint of a
                                     time-sharded forward, where dy exists only on the own frames */
} msl_dwconv_geometry;

#define MSL_EPI_NONE 0      /* y = conv(x) + bias + bias2 */
#define MSL_EPI_GELU 1      /* y = gelu_erf(conv(x) + bias) */
#define MSL_EPI_GELU_GRAD 2 /* y = aux * gelu_erf'(conv(x) + bias)  (offset_net backward) */
#define MSL_EPI_ACCUM 3     /* y += conv(x) + bias + bias2  (float32 y only) */

/* y[out frames] = epilogue(conv(x[in frames])).  bias, bias2 float32 [C] or NULL.  geom->dtype is
 * the element type of x; y_dtype (MSL_DTYPE_*) that of y and aux (a bf16 input can produce a float32
 * GELU-gradient). */
int msl_dwconv3d_fwd(const msl_dwconv_geometry* geom, const void* x, int64_t x_ld,
                     const float* weight, const float* bias, const float* bias2, int32_t epilogue,
                     const void* aux, int64_t aux_ld, void* y, int64_t y_ld, int32_t y_dtype,
                     void* stream);

/* dx[out frames] = conv_transpose(dy[in frames]) (gradient w.r.t. the conv input). */
int msl_dwconv3d_bwd_data(const msl_dwconv_geometry* geom, const void* dy, int64_t dy_ld,
                          const float* weight, void* dx, int64_t dx_ld, void* stream);

/* dx[out frames] (float32) += conv_transpose(dy[in frames]): the input gradient added into a float32
 * buffer that already holds the other branches' terms (no temporary, no separate add pass). */
int msl_dwconv3d_bwd_data_acc(const msl_dwconv_geometry* geom, const void* dy, int64_t dy_ld,
                              const float* weight, float* dx, int64_t dx_ld, void* stream);

/* dweight[kt*kh*kw, C] += sum over dy positions (out frames) of dy * shifted x (in frames);
 * dbias[C] += sum of dy (dbias may be NULL).  Accumulates: the caller clears.  geom->dtype is the
 * element type of x, dy_dtype that of dy. */
int msl_dwconv3d_bwd_weight(const msl_dwconv_geometry* geom, const void* dy, int64_t dy_ld,
                            int32_t dy_dtype, const void* x, int64_t x_ld, float* dweight,
                            float* dbias, void* stream);

/* ----------------------------------------------------------------------------------------------
 * Utilities
 * ---------------------------------------------------------------------------------------------- */
/* Per-axis maximum |offset*offset_scale| (in the reference's raw offset units) over a float32
 * offset tensor [rows, >=heads*taps*3] (row stride ld): out3[0..2] = max over channels 0, 1, 2 of
 * every tap.  bias (float32 [heads*taps*3] or NULL) is added to every row first, as in offset_bias
 * of msl_dsa_fwd_io.  out3 (device, float32[3]) must be zeroed by the caller; values are max-accumulated.
 * Used to size the time halo of the sharded path. */
int msl_offsets_absmax(const float* offsets, int64_t rows, int64_t ld, const float* bias, int32_t heads,
                       int32_t taps, float offset_scale, float* out3, void* stream);

/* Element-type conversion float32 -> dtype of a [rows, cols] matrix (row strides in elements). */
int msl_convert_f32(const float* src, int64_t src_ld, void* dst, int64_t dst_ld, int32_t dtype,
                    int64_t rows, int64_t cols, void* stream);

int32_t msl_abi_version(void);
/* Kernel launches issued by this library since it was loaded (all threads). */
uint64_t msl_launch_count(void);
/* Description of the last error returned on the calling thread ("" if none). */
const char* msl_last_error(void);

/* ----------------------------------------------------------------------------------------------
 * Host-side optimizer kernels of the CPU-master trainer (megaslide_b200/stream.py).  Plain host
 * memory, multi-threaded (OpenMP), no GPU involvement.  They replace torch.optim.AdamW and the
 * per-parameter gradient accumulation of the reference's CPUMasterVideoDiT
 * (infinity/video/trainer.py:66-72, 176-221, 575-599).
 * ---------------------------------------------------------------------------------------------- */

/* dst[i] = (overwrite ? 0 : dst[i]) + src[i] for n float32 dst elements; src is float32 or bf16
 * (src_dtype MSL_DTYPE_*).  *sumsq (optional) receives sum(dst^2) in double precision. */
int msl_host_accumulate(float* dst, const void* src, int32_t src_dtype, int64_t n, int32_t overwrite,
                        double* sumsq);

/* One AdamW step (torch.optim.AdamW's update: decoupled weight decay, bias-corrected moments) over n
 * float32 elements: g is scaled by grad_scale (gradient clipping) first; step = the step number
 * after this update (>= 1).  stage (optional, MSL_DTYPE_F32 or MSL_DTYPE_BF16) receives the updated
 * parameters in the compute dtype (bf16 rounded to nearest even) in the same pass. */
int msl_host_adamw(float* p, float* m, float* v, const float* g, int64_t n, float lr, float beta1, float beta2,
                   float eps, float weight_decay, int64_t step, float grad_scale, void* stage,
                   int32_t stage_dtype);

#ifdef __cplusplus
}
#endif
#endif /* MEGASLIDE_B200_H */
