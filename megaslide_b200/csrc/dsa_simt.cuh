// CUDA-core ("gather") deformable slide attention for ONE (sample, query, head), as warp-level device
// functions: the bodies of the CUDA-core kernels (dsa_attn.cu) and the fallback of the tensor-core
// kernels for a tile whose key envelope their sample records cannot encode.
//
// One warp owns one (sample b, query row, head).  Its 32 lanes are split as 8 trilinear corners x
// 4 channel slots: lane = corner*4 + slot, corner bits (dt, dh, dw).  For every window sample the
// warp computes the clamped voxel coordinate once (lane j of a 32-sample batch computes sample j,
// then it is broadcast), each lane fetches its corner's K (and V) row in 16-byte chunks of its
// channel slot, and a warp reduction turns the 32 partial products into the sample's score.  The
// softmax is an online (running max) softmax in base 2, so a query's samples are never stored.
// All 32 lanes of the warp must call these functions together.
//
// Reference semantics (infinity/video/attention.py): grid construction :113-127 and :194-238,
// trilinear border sampling :240-273, scores / softmax / dropout / value sum :147-186, extra keys
// :159-173.
#pragma once

#include <math.h>

#include "dsa_attn.cuh"
#include "msl_common.cuh"

namespace msl {

__device__ __forceinline__ uint64_t softmax_index(const AttnParams& P, int b, int tg, int h, int w,
                                                  int head, int j) {
  const uint64_t q = ((static_cast<uint64_t>(b) * P.T + tg) * P.H + h) * P.W + w;
  return (q * P.nh + head) * static_cast<uint64_t>(P.K + P.G) + j;
}

struct QueryPos {
  int b, head, tg, h, w;
  long long r;  // query row within this call's frames
};

template <typename T, int VEC, int MAXC>
__device__ __forceinline__ void fwd_query(const AttnParams& P, const QueryPos& qp) {
  const int lane = threadIdx.x & 31;
  const int corner = lane >> 2, slot = lane & 3;
  const int cdt = corner >> 2, cdh = (corner >> 1) & 1, cdw = corner & 1;
  const int nchunk = P.d / VEC;

  const T* qrow = static_cast<const T*>(P.q) + (qp.b * P.Nq + qp.r) * P.q_ld + qp.head * P.d;
  float qf[MAXC][VEC], acc[MAXC][VEC];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int ck = slot + 4 * i;
    if (ck < nchunk) {
      Chunk<T, VEC>::load(qrow + ck * VEC, qf[i]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) qf[i][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[i][e] = 0.f;
  }

  const T* kbase = static_cast<const T*>(P.k) + static_cast<long long>(qp.b) * P.Nkv * P.k_ld + qp.head * P.d;
  const T* vbase = static_cast<const T*>(P.v) + static_cast<long long>(qp.b) * P.Nkv * P.v_ld + qp.head * P.d;
  const float* orow = P.offsets + (qp.b * P.Nq + qp.r) * P.off_ld + static_cast<long long>(qp.head) * P.K * 3;
  const SampleGeom sg{P.T, P.H, P.W, P.kt, P.kh, P.kw, P.oscale};

  float m2 = -INFINITY, l = 0.f;
  bool miss = false;
  for (int j0 = 0; j0 < P.K; j0 += 32) {
    float mpt = 0.f, mph = 0.f, mpw = 0.f;
    const int jl = j0 + lane;
    if (jl < P.K) {
      float o0, o1, o2;
      load_off3(P, orow, qp.head, jl, o0, o1, o2);
      sample_coords(sg, qp.tg, qp.h, qp.w, jl, o0, o1, o2, mpt, mph, mpw);
    }
    const int ns = min(32, P.K - j0);
    for (int jj = 0; jj < ns; ++jj) {
      const float pt = __shfl_sync(kFull, mpt, jj);
      const float ph = __shfl_sync(kFull, mph, jj);
      const float pw = __shfl_sync(kFull, mpw, jj);
      const int t0 = static_cast<int>(floorf(pt)), h0 = static_cast<int>(floorf(ph)), w0 = static_cast<int>(floorf(pw));
      const int tc = t0 + cdt, hc = h0 + cdh, wc = w0 + cdw;
      bool inb = (tc < P.T) && (hc < P.H) && (wc < P.W);
      const int tk = tc - P.kv_frame0;
      if (inb && (tk < 0 || tk >= P.kv_frames)) {
        miss = true;
        inb = false;
      }
      const long long krow = (static_cast<long long>(tk) * P.H + hc) * P.W + wc;
      float wgt = 0.f, part = 0.f;
      if (inb) {
        wgt = __fmul_rn(__fmul_rn(axis_weight(pw, w0, cdw), axis_weight(ph, h0, cdh)), axis_weight(pt, t0, cdt));
        const T* kp = kbase + krow * P.k_ld;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
          const int ck = slot + 4 * i;
          if (ck < nchunk) {
            float kv[VEC];
            Chunk<T, VEC>::load(kp + ck * VEC, kv);
#pragma unroll
            for (int e = 0; e < VEC; ++e) part = fmaf(qf[i][e], kv[e], part);
          }
        }
        part *= wgt;
      }
      const float s2 = warp_sum(part) * P.scale_log2;
      if (s2 > m2) {
        const float alpha = exp2f(m2 - s2);
        l *= alpha;
#pragma unroll
        for (int i = 0; i < MAXC; ++i)
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[i][e] *= alpha;
        m2 = s2;
      }
      const float p = exp2f(s2 - m2);
      l += p;
      float pv = p;
      if (P.drop_thresh &&
          !dropout_keep(P.seed, softmax_index(P, qp.b, qp.tg, qp.h, qp.w, qp.head, j0 + jj), P.drop_thresh))
        pv = 0.f;
      else if (P.drop_thresh)
        pv = p * P.drop_keep_scale;
      if (inb && pv != 0.f) {
        const float coef = pv * wgt;
        const T* vp = vbase + krow * P.v_ld;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
          const int ck = slot + 4 * i;
          if (ck < nchunk) {
            float vv[VEC];
            Chunk<T, VEC>::load(vp + ck * VEC, vv);
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[i][e] = fmaf(coef, vv[e], acc[i][e]);
          }
        }
      }
    }
  }

  // Extra keys / values shared by every query of the sample (attention.py:159-173): one exact
  // "corner" each, handled by the corner-0 lanes.
  for (int g = 0; g < P.G; ++g) {
    const long long erow = (static_cast<long long>(qp.b) * P.G + g) * P.e_ld + qp.head * P.d;
    float part = 0.f;
    if (corner == 0) {
      const T* kp = static_cast<const T*>(P.ek) + erow;
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int ck = slot + 4 * i;
        if (ck < nchunk) {
          float kv[VEC];
          Chunk<T, VEC>::load(kp + ck * VEC, kv);
#pragma unroll
          for (int e = 0; e < VEC; ++e) part = fmaf(qf[i][e], kv[e], part);
        }
      }
    }
    const float s2 = warp_sum(part) * P.scale_log2;
    if (s2 > m2) {
      const float alpha = exp2f(m2 - s2);
      l *= alpha;
#pragma unroll
      for (int i = 0; i < MAXC; ++i)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[i][e] *= alpha;
      m2 = s2;
    }
    const float p = exp2f(s2 - m2);
    l += p;
    float pv = p;
    if (P.drop_thresh)
      pv = dropout_keep(P.seed, softmax_index(P, qp.b, qp.tg, qp.h, qp.w, qp.head, P.K + g), P.drop_thresh)
               ? p * P.drop_keep_scale
               : 0.f;
    if (corner == 0 && pv != 0.f) {
      const T* vp = static_cast<const T*>(P.ev) + erow;
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int ck = slot + 4 * i;
        if (ck < nchunk) {
          float vv[VEC];
          Chunk<T, VEC>::load(vp + ck * VEC, vv);
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[i][e] = fmaf(pv, vv[e], acc[i][e]);
        }
      }
    }
  }

  // Sum the 8 corner partial accumulators of each channel slot.
#pragma unroll
  for (int i = 0; i < MAXC; ++i)
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float v = acc[i][e];
      v += __shfl_xor_sync(kFull, v, 4);
      v += __shfl_xor_sync(kFull, v, 8);
      v += __shfl_xor_sync(kFull, v, 16);
      acc[i][e] = v;
    }
  const float inv_l = 1.f / l;
  if (corner == 0) {
    T* orow_out = static_cast<T*>(P.out) + (qp.b * P.Nq + qp.r) * P.out_ld + qp.head * P.d;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int ck = slot + 4 * i;
      if (ck < nchunk) {
        float o[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = acc[i][e] * inv_l;
        Chunk<T, VEC>::store(orow_out + ck * VEC, o);
      }
    }
  }
  if (lane == 0) P.lse[(static_cast<long long>(qp.b) * P.nh + qp.head) * P.Nq + qp.r] = m2 + log2f(l);
  if (__any_sync(kFull, miss) && lane == 0 && P.status) atomicOr(P.status, MSL_STATUS_HALO_MISS);
}

template <typename T, int VEC, int MAXC>
__device__ __forceinline__ void bwd_query(const AttnParams& P, const QueryPos& qp) {
  const int lane = threadIdx.x & 31;
  const int corner = lane >> 2, slot = lane & 3;
  const int cdt = corner >> 2, cdh = (corner >> 1) & 1, cdw = corner & 1;
  const float sgx = cdw ? 1.f : -1.f, sgy = cdh ? 1.f : -1.f, sgz = cdt ? 1.f : -1.f;
  const int nchunk = P.d / VEC;
  const long long qrow_i = qp.b * P.Nq + qp.r;

  const T* qrow = static_cast<const T*>(P.q) + qrow_i * P.q_ld + qp.head * P.d;
  const T* dorow = static_cast<const T*>(P.dout) + qrow_i * P.dout_ld + qp.head * P.d;
  const T* oorow = static_cast<const T*>(P.out) + qrow_i * P.out_ld + qp.head * P.d;
  float qf[MAXC][VEC], dof[MAXC][VEC], dqa[MAXC][VEC];
  float dpart = 0.f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int ck = slot + 4 * i;
    if (ck < nchunk) {
      Chunk<T, VEC>::load(qrow + ck * VEC, qf[i]);
      Chunk<T, VEC>::load(dorow + ck * VEC, dof[i]);
      float ov[VEC];
      Chunk<T, VEC>::load(oorow + ck * VEC, ov);
#pragma unroll
      for (int e = 0; e < VEC; ++e) dpart = fmaf(ov[e], dof[i][e], dpart);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) qf[i][e] = dof[i][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) dqa[i][e] = 0.f;
  }
  // D = dout . out  (softmax backward row term); every corner group holds the same partials.
  dpart += __shfl_xor_sync(kFull, dpart, 1);
  dpart += __shfl_xor_sync(kFull, dpart, 2);
  const float Dterm = dpart;
  const float lse2 = P.lse[(static_cast<long long>(qp.b) * P.nh + qp.head) * P.Nq + qp.r];

  const T* kbase = static_cast<const T*>(P.k) + static_cast<long long>(qp.b) * P.Nkv * P.k_ld + qp.head * P.d;
  const T* vbase = static_cast<const T*>(P.v) + static_cast<long long>(qp.b) * P.Nkv * P.v_ld + qp.head * P.d;
  float* dkbase = P.dk_acc + static_cast<long long>(qp.b) * P.Nkv * P.acc_ld + qp.head * P.d;
  float* dvbase = P.dv_acc + static_cast<long long>(qp.b) * P.Nkv * P.acc_ld + qp.head * P.d;
  const float* orow = P.offsets + qrow_i * P.off_ld + static_cast<long long>(qp.head) * P.K * 3;
  const long long dorow_off = qrow_i * P.doff_ld + static_cast<long long>(qp.head) * P.K * 3;
  const SampleGeom sg{P.T, P.H, P.W, P.kt, P.kh, P.kw, P.oscale};
  bool miss = false;

  for (int j0 = 0; j0 < P.K; j0 += 32) {
    float mpt = 0.f, mph = 0.f, mpw = 0.f;
    const int jl = j0 + lane;
    if (jl < P.K) {
      float o0, o1, o2;
      load_off3(P, orow, qp.head, jl, o0, o1, o2);
      sample_coords(sg, qp.tg, qp.h, qp.w, jl, o0, o1, o2, mpt, mph, mpw);
    }
    float my_gw = 0.f, my_gh = 0.f, my_gt = 0.f;
    const int ns = min(32, P.K - j0);
    for (int jj = 0; jj < ns; ++jj) {
      const float pt = __shfl_sync(kFull, mpt, jj);
      const float ph = __shfl_sync(kFull, mph, jj);
      const float pw = __shfl_sync(kFull, mpw, jj);
      const int t0 = static_cast<int>(floorf(pt)), h0 = static_cast<int>(floorf(ph)), w0 = static_cast<int>(floorf(pw));
      const int tc = t0 + cdt, hc = h0 + cdh, wc = w0 + cdw;
      bool inb = (tc < P.T) && (hc < P.H) && (wc < P.W);
      const int tk = tc - P.kv_frame0;
      if (inb && (tk < 0 || tk >= P.kv_frames)) {
        miss = true;
        inb = false;
      }
      const long long krow = (static_cast<long long>(tk) * P.H + hc) * P.W + wc;
      const float ax = axis_weight(pw, w0, cdw), ay = axis_weight(ph, h0, cdh), az = axis_weight(pt, t0, cdt);
      float wgt = 0.f, kd = 0.f, vd = 0.f;
      float kr[MAXC][VEC];
      if (inb) {
        wgt = __fmul_rn(__fmul_rn(ax, ay), az);
        const T* kp = kbase + krow * P.k_ld;
        const T* vp = vbase + krow * P.v_ld;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
          const int ck = slot + 4 * i;
          if (ck < nchunk) {
            float vv[VEC];
            Chunk<T, VEC>::load(kp + ck * VEC, kr[i]);
            Chunk<T, VEC>::load(vp + ck * VEC, vv);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              kd = fmaf(qf[i][e], kr[i][e], kd);
              vd = fmaf(dof[i][e], vv[e], vd);
            }
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) kr[i][e] = 0.f;
          }
        }
      }
      // full per-corner dots (q.k_c, dout.v_c), identical on the corner's 4 slot lanes
      kd += __shfl_xor_sync(kFull, kd, 1);
      kd += __shfl_xor_sync(kFull, kd, 2);
      vd += __shfl_xor_sync(kFull, vd, 1);
      vd += __shfl_xor_sync(kFull, vd, 2);
      float sk = wgt * kd, sv = wgt * vd;
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        sk += __shfl_xor_sync(kFull, sk, o);
        sv += __shfl_xor_sync(kFull, sv, o);
      }
      const float p = exp2f(sk * P.scale_log2 - lse2);
      float ks = 1.f;
      if (P.drop_thresh)
        ks = dropout_keep(P.seed, softmax_index(P, qp.b, qp.tg, qp.h, qp.w, qp.head, j0 + jj), P.drop_thresh)
                 ? P.drop_keep_scale
                 : 0.f;
      const float pv = p * ks;          // weight applied to the sampled value
      const float ds = p * (sv * ks - Dterm);
      const float dsq = ds * P.scale;   // dL / d(q . k_sample)
      if (inb) {
        const float cq = dsq * wgt, cv = pv * wgt;
        float* dkp = dkbase + krow * P.acc_ld;
        float* dvp = dvbase + krow * P.acc_ld;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
          const int ck = slot + 4 * i;
          if (ck < nchunk) {
            float tk_[VEC], tv_[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              dqa[i][e] = fmaf(cq, kr[i][e], dqa[i][e]);
              tk_[e] = cq * qf[i][e];
              tv_[e] = cv * dof[i][e];
            }
            atomic_add_chunk<VEC>(dkp + ck * VEC, tk_);
            if (cv != 0.f) atomic_add_chunk<VEC>(dvp + ck * VEC, tv_);
          }
        }
      }
      // d loss / d voxel coordinate (grid_sampler_3d_backward's gix/giy/giz before the
      // clip multiplier), summed over the corners this sample touches.
      const float gcor = inb ? fmaf(dsq, kd, pv * vd) : 0.f;
      float gw_ = sgx * ay * az * gcor, gh_ = ax * sgy * az * gcor, gt_ = ax * ay * sgz * gcor;
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        gw_ += __shfl_xor_sync(kFull, gw_, o);
        gh_ += __shfl_xor_sync(kFull, gh_, o);
        gt_ += __shfl_xor_sync(kFull, gt_, o);
      }
      if (lane == jj) {
        my_gw = gw_ * clip_grad_mult(pw, P.W);
        my_gh = gh_ * clip_grad_mult(ph, P.H);
        my_gt = gt_ * clip_grad_mult(pt, P.T);
      }
    }
    if (jl < P.K) {
      // channel 0 moved grid x (W) after division by (T-1); channel 2 moved grid z (T) after
      // division by (W-1) (attention.py:118-127).
      store_doff(P, dorow_off + jl * 3 + 0, (P.T > 1) ? __fdiv_rn(my_gw, static_cast<float>(P.T - 1)) * P.oscale : 0.f);
      store_doff(P, dorow_off + jl * 3 + 1, (P.H > 1) ? __fdiv_rn(my_gh, static_cast<float>(P.H - 1)) * P.oscale : 0.f);
      store_doff(P, dorow_off + jl * 3 + 2, (P.W > 1) ? __fdiv_rn(my_gt, static_cast<float>(P.W - 1)) * P.oscale : 0.f);
    }
  }

  for (int g = 0; g < P.G; ++g) {
    const long long erow = (static_cast<long long>(qp.b) * P.G + g) * P.e_ld + qp.head * P.d;
    float kd = 0.f, vd = 0.f;
    float kr[MAXC][VEC];
    if (corner == 0) {
      const T* kp = static_cast<const T*>(P.ek) + erow;
      const T* vp = static_cast<const T*>(P.ev) + erow;
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int ck = slot + 4 * i;
        if (ck < nchunk) {
          float vv[VEC];
          Chunk<T, VEC>::load(kp + ck * VEC, kr[i]);
          Chunk<T, VEC>::load(vp + ck * VEC, vv);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            kd = fmaf(qf[i][e], kr[i][e], kd);
            vd = fmaf(dof[i][e], vv[e], vd);
          }
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) kr[i][e] = 0.f;
        }
      }
    }
    kd = warp_sum(kd);
    vd = warp_sum(vd);
    const float p = exp2f(kd * P.scale_log2 - lse2);
    float ks = 1.f;
    if (P.drop_thresh)
      ks = dropout_keep(P.seed, softmax_index(P, qp.b, qp.tg, qp.h, qp.w, qp.head, P.K + g), P.drop_thresh)
               ? P.drop_keep_scale
               : 0.f;
    const float pv = p * ks;
    const float dsq = p * (vd * ks - Dterm) * P.scale;
    if (corner == 0) {
#pragma unroll
      for (int i = 0; i < MAXC; ++i)
#pragma unroll
        for (int e = 0; e < VEC; ++e) dqa[i][e] = fmaf(dsq, kr[i][e], dqa[i][e]);
    }
    if (lane == 0) {
      const long long xi = ((static_cast<long long>(qp.b) * P.nh + qp.head) * P.Nq + qp.r) * P.G + g;
      P.extra_ds[xi] = dsq;
      P.extra_p[xi] = pv;
    }
  }

#pragma unroll
  for (int i = 0; i < MAXC; ++i)
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float v = dqa[i][e];
      v += __shfl_xor_sync(kFull, v, 4);
      v += __shfl_xor_sync(kFull, v, 8);
      v += __shfl_xor_sync(kFull, v, 16);
      dqa[i][e] = v;
    }
  if (corner == 0) {
    T* dqrow = static_cast<T*>(P.dq) + qrow_i * P.dq_ld + qp.head * P.d;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int ck = slot + 4 * i;
      if (ck < nchunk) Chunk<T, VEC>::store(dqrow + ck * VEC, dqa[i]);
    }
  }
  if (__any_sync(kFull, miss) && lane == 0 && P.status) atomicOr(P.status, MSL_STATUS_HALO_MISS);
}

}  // namespace msl
