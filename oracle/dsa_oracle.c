/*
 * CPU oracle for the 3D deformable slide attention hot path.  TEST INFRASTRUCTURE ONLY: it is
 * the checker that tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * compare against; the product path (megaslide_b200) never links or calls it.
 *
 * It restates, in plain C, the algorithm of the reference module
 * infinity/video/attention.py (jasonliu0704/megaslide):
 *   - base grid 2a/max(S-1,1)-1 in float32                     attention.py:208-236
 *   - offset normalisation with the channel/axis swap           attention.py:113-127
 *       (channel 0 / (T-1) moves grid x = W, channel 1 / (H-1) moves y = H,
 *        channel 2 / (W-1) moves z = T)
 *   - grid_sample(mode='bilinear' (trilinear on 5-D), padding_mode='border',
 *       align_corners=False) of K and V                          attention.py:240-273
 *       unnormalise p = ((g+1)*S-1)/2, clamp to [0,S-1], 8 corners with weights
 *       ((i0+1)-p or p-i0 per axis), out-of-volume corners contribute 0; the
 *       coordinate gradient is 0 on/beyond the border (the grid_sample contract in
 *       PyTorch's ATen/native/GridSampler.h: clip_coordinates_set_grad)
 *   - scores q.k/sqrt(d), softmax over the window (+ G extra keys), dropout,
 *       weighted value sum                                        attention.py:147-186
 *   - depthwise 3D convolution, zero padding k//2                attention.py:58-74
 * Coordinates are computed in float32 with the reference's operation order (this file is
 * compiled with -ffp-contract=off so no step is fused); everything else accumulates in
 * double precision.
 *
 * Dropout uses the same counter-based SplitMix64 keep rule as the CUDA kernels, so the
 * oracle reproduces their masks exactly (the reference draws its mask from torch's RNG,
 * which no other implementation can reproduce).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct oracle_geom {
  int32_t B, T, H, W, nh, d, kt, kh, kw, G;
  double softmax_scale;
  float offset_scale;
  float dropout_p;
  uint64_t dropout_seed;
} oracle_geom;

static float base_grid(int a, int S) {
  const float den = (float)(S > 1 ? S - 1 : 1);
  const float two_a = (float)(2 * a);
  const float q = two_a / den;
  return q - 1.0f;
}

static float unnorm_clip(float g, int S) {
  const float t1 = g + 1.0f;
  const float t2 = t1 * (float)S;
  const float t3 = t2 - 1.0f;
  const float v = t3 / 2.0f;
  const float hi = (float)(S - 1);
  const float lo = (v < 0.f) ? 0.f : v;
  return (lo < hi) ? lo : hi;
}

static double clip_mult(float p, int S) { return (p > 0.f && p < (float)(S - 1)) ? 0.5 * (double)S : 0.0; }

static void coords(const oracle_geom* g, int t, int h, int w, int j, const float* o, float* pt, float* ph,
                   float* pw) {
  const int khw = g->kh * g->kw;
  const int it = j / khw, rem = j % khw, ih = rem / g->kw, iw = rem % g->kw;
  float gx = base_grid(w + iw - g->kw / 2, g->W);
  float gy = base_grid(h + ih - g->kh / 2, g->H);
  float gz = base_grid(t + it - g->kt / 2, g->T);
  const float o0 = o[0] * g->offset_scale, o1 = o[1] * g->offset_scale, o2 = o[2] * g->offset_scale;
  if (g->T > 1) gx = gx + o0 / (float)(g->T - 1);
  if (g->H > 1) gy = gy + o1 / (float)(g->H - 1);
  if (g->W > 1) gz = gz + o2 / (float)(g->W - 1);
  *pw = unnorm_clip(gx, g->W);
  *ph = unnorm_clip(gy, g->H);
  *pt = unnorm_clip(gz, g->T);
}

static uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

static uint32_t drop_threshold(float p) {
  if (!(p > 0.f)) return 0;
  const double th = (double)p * 4294967296.0;
  uint32_t t = th >= 4294967295.0 ? 0xffffffffu : (uint32_t)th;
  return t ? t : 1;
}

/* keep factor (0 or 1/(1-p)) of softmax weight j of the query (b, t, h, w, head) */
static double keep_factor(const oracle_geom* g, uint32_t thr, int b, int t, int h, int w, int head, int j) {
  if (!thr) return 1.0;
  const uint64_t q = (((uint64_t)b * g->T + t) * g->H + h) * g->W + w;
  const uint64_t idx = (q * g->nh + head) * (uint64_t)(g->kt * g->kh * g->kw + g->G) + j;
  const uint64_t r = splitmix64(g->dropout_seed ^ (idx * 0xD1B54A32D192ED03ull));
  if ((uint32_t)(r >> 32) < thr) return 0.0;
  return (double)(1.0f / (1.0f - g->dropout_p));
}

typedef struct corner8 {
  int valid[8];
  long row[8];
  double w[8];
  double dwx[8], dwy[8], dwz[8]; /* d weight / d p{x,y,z} */
} corner8;

static void make_corners(const oracle_geom* g, float pt, float ph, float pw, corner8* c) {
  const int t0 = (int)floorf(pt), h0 = (int)floorf(ph), w0 = (int)floorf(pw);
  for (int k = 0; k < 8; ++k) {
    const int dt = k >> 2, dh = (k >> 1) & 1, dw = k & 1;
    const int tc = t0 + dt, hc = h0 + dh, wc = w0 + dw;
    const double ax = dw ? (double)pw - w0 : (double)(w0 + 1) - pw;
    const double ay = dh ? (double)ph - h0 : (double)(h0 + 1) - ph;
    const double az = dt ? (double)pt - t0 : (double)(t0 + 1) - pt;
    c->valid[k] = tc < g->T && hc < g->H && wc < g->W;
    c->row[k] = ((long)tc * g->H + hc) * g->W + wc;
    c->w[k] = ax * ay * az;
    c->dwx[k] = (dw ? 1.0 : -1.0) * ay * az;
    c->dwy[k] = ax * (dh ? 1.0 : -1.0) * az;
    c->dwz[k] = ax * ay * (dt ? 1.0 : -1.0);
  }
}

/* Forward.  q, out: [B, N, C]; k, v: [B, N, C]; off: float32 [B, N, nh*K*3];
 * ek, ev: [B, G, C] (or NULL when G == 0); lse: natural-log log-sum-exp [B, nh, N]. */
void oracle_dsa_fwd(const oracle_geom* g, const double* q, const double* k, const double* v, const float* off,
                    const double* ek, const double* ev, double* out, double* lse) {
  const int K = g->kt * g->kh * g->kw, G = g->G, d = g->d, nh = g->nh;
  const long N = (long)g->T * g->H * g->W, C = (long)nh * d;
  const uint32_t thr = drop_threshold(g->dropout_p);
  const long items = (long)g->B * nh * N;
#pragma omp parallel
  {
    double* s = (double*)malloc(sizeof(double) * (K + G));
    double* ks = (double*)malloc(sizeof(double) * d);
    corner8* cs = (corner8*)malloc(sizeof(corner8) * K);
#pragma omp for schedule(dynamic, 64)
    for (long it = 0; it < items; ++it) {
      const long n = it % N;
      const int head = (int)((it / N) % nh), b = (int)(it / N / nh);
      const int t = (int)(n / (g->H * g->W)), h = (int)((n / g->W) % g->H), w = (int)(n % g->W);
      const double* qr = q + ((long)b * N + n) * C + head * d;
      const float* orow = off + ((long)b * N + n) * (long)nh * K * 3 + (long)head * K * 3;
      double m = -INFINITY;
      for (int j = 0; j < K; ++j) {
        float pt, ph, pw;
        coords(g, t, h, w, j, orow + 3 * j, &pt, &ph, &pw);
        make_corners(g, pt, ph, pw, &cs[j]);
        for (int i = 0; i < d; ++i) ks[i] = 0.0;
        for (int c = 0; c < 8; ++c) {
          if (!cs[j].valid[c]) continue;
          const double* kr = k + ((long)b * N + cs[j].row[c]) * C + head * d;
          for (int i = 0; i < d; ++i) ks[i] += cs[j].w[c] * kr[i];
        }
        double dot = 0.0;
        for (int i = 0; i < d; ++i) dot += qr[i] * ks[i];
        s[j] = dot * g->softmax_scale;
        if (s[j] > m) m = s[j];
      }
      for (int e = 0; e < G; ++e) {
        const double* kr = ek + ((long)b * G + e) * C + head * d;
        double dot = 0.0;
        for (int i = 0; i < d; ++i) dot += qr[i] * kr[i];
        s[K + e] = dot * g->softmax_scale;
        if (s[K + e] > m) m = s[K + e];
      }
      double l = 0.0;
      for (int j = 0; j < K + G; ++j) l += exp(s[j] - m);
      double* orow_out = out + ((long)b * N + n) * C + head * d;
      for (int i = 0; i < d; ++i) orow_out[i] = 0.0;
      for (int j = 0; j < K; ++j) {
        const double p = exp(s[j] - m) / l * keep_factor(g, thr, b, t, h, w, head, j);
        if (p == 0.0) continue;
        for (int c = 0; c < 8; ++c) {
          if (!cs[j].valid[c]) continue;
          const double* vr = v + ((long)b * N + cs[j].row[c]) * C + head * d;
          const double pw_ = p * cs[j].w[c];
          for (int i = 0; i < d; ++i) orow_out[i] += pw_ * vr[i];
        }
      }
      for (int e = 0; e < G; ++e) {
        const double p = exp(s[K + e] - m) / l * keep_factor(g, thr, b, t, h, w, head, K + e);
        const double* vr = ev + ((long)b * G + e) * C + head * d;
        for (int i = 0; i < d; ++i) orow_out[i] += p * vr[i];
      }
      lse[((long)b * nh + head) * N + n] = m + log(l);
    }
    free(s);
    free(ks);
    free(cs);
  }
}

/* Backward of oracle_dsa_fwd.  Outputs are overwritten: dq [B,N,C], dk, dv [B,N,C],
 * doff float64 [B, N, nh*K*3] (gradient w.r.t. the raw offsets), dek, dev [B,G,C]. */
void oracle_dsa_bwd(const oracle_geom* g, const double* q, const double* k, const double* v, const float* off,
                    const double* ek, const double* ev, const double* dout, double* dq, double* dk, double* dv,
                    double* doff, double* dek, double* dev) {
  const int K = g->kt * g->kh * g->kw, G = g->G, d = g->d, nh = g->nh;
  const long N = (long)g->T * g->H * g->W, C = (long)nh * d;
  const uint32_t thr = drop_threshold(g->dropout_p);
  const long items = (long)g->B * nh * N;
  const long kvn = (long)g->B * N * C, en = (long)g->B * G * C;
  memset(dk, 0, sizeof(double) * kvn);
  memset(dv, 0, sizeof(double) * kvn);
  if (G > 0) {
    memset(dek, 0, sizeof(double) * en);
    memset(dev, 0, sizeof(double) * en);
  }
#pragma omp parallel
  {
    double* pdk = (double*)calloc(kvn, sizeof(double));
    double* pdv = (double*)calloc(kvn, sizeof(double));
    double* pdek = G > 0 ? (double*)calloc(en, sizeof(double)) : NULL;
    double* pdev = G > 0 ? (double*)calloc(en, sizeof(double)) : NULL;
    double* s = (double*)malloc(sizeof(double) * (K + G));
    double* kdc = (double*)malloc(sizeof(double) * K * 8);
    double* vdc = (double*)malloc(sizeof(double) * K * 8);
    double* dpv = (double*)malloc(sizeof(double) * (K + G));
    double* osum = (double*)malloc(sizeof(double) * d);
    corner8* cs = (corner8*)malloc(sizeof(corner8) * K);
    float* pts = (float*)malloc(sizeof(float) * 3 * K);
#pragma omp for schedule(dynamic, 64)
    for (long it = 0; it < items; ++it) {
      const long n = it % N;
      const int head = (int)((it / N) % nh), b = (int)(it / N / nh);
      const int t = (int)(n / (g->H * g->W)), h = (int)((n / g->W) % g->H), w = (int)(n % g->W);
      const long qrow = ((long)b * N + n) * C + head * d;
      const double* qr = q + qrow;
      const double* dor = dout + qrow;
      const float* orow = off + ((long)b * N + n) * (long)nh * K * 3 + (long)head * K * 3;
      double* doffr = doff + ((long)b * N + n) * (long)nh * K * 3 + (long)head * K * 3;
      double m = -INFINITY;
      for (int j = 0; j < K; ++j) {
        float pt, ph, pw;
        coords(g, t, h, w, j, orow + 3 * j, &pt, &ph, &pw);
        pts[3 * j] = pt; pts[3 * j + 1] = ph; pts[3 * j + 2] = pw;
        make_corners(g, pt, ph, pw, &cs[j]);
        double sj = 0.0, dpj = 0.0;
        for (int c = 0; c < 8; ++c) {
          double kd = 0.0, vd = 0.0;
          if (cs[j].valid[c]) {
            const double* kr = k + ((long)b * N + cs[j].row[c]) * C + head * d;
            const double* vr = v + ((long)b * N + cs[j].row[c]) * C + head * d;
            for (int i = 0; i < d; ++i) {
              kd += qr[i] * kr[i];
              vd += dor[i] * vr[i];
            }
          }
          kdc[j * 8 + c] = kd;
          vdc[j * 8 + c] = vd;
          sj += cs[j].w[c] * kd;
          dpj += cs[j].w[c] * vd;
        }
        s[j] = sj * g->softmax_scale;
        dpv[j] = dpj;
        if (s[j] > m) m = s[j];
      }
      for (int e = 0; e < G; ++e) {
        const double* kr = ek + ((long)b * G + e) * C + head * d;
        const double* vr = ev + ((long)b * G + e) * C + head * d;
        double kd = 0.0, vd = 0.0;
        for (int i = 0; i < d; ++i) {
          kd += qr[i] * kr[i];
          vd += dor[i] * vr[i];
        }
        s[K + e] = kd * g->softmax_scale;
        dpv[K + e] = vd;
        if (s[K + e] > m) m = s[K + e];
      }
      double l = 0.0;
      for (int j = 0; j < K + G; ++j) l += exp(s[j] - m);
      /* D = sum_j p_j * keep_j * dp_j  (= dout . out) */
      double D = 0.0;
      for (int j = 0; j < K + G; ++j) {
        const double kf = keep_factor(g, thr, b, t, h, w, head, j);
        D += exp(s[j] - m) / l * kf * dpv[j];
      }
      for (int i = 0; i < d; ++i) osum[i] = 0.0;
      for (int j = 0; j < K; ++j) {
        const double p = exp(s[j] - m) / l;
        const double kf = keep_factor(g, thr, b, t, h, w, head, j);
        const double ds = p * (dpv[j] * kf - D);
        const double dsq = ds * g->softmax_scale;
        const double pv = p * kf;
        double gx = 0.0, gy = 0.0, gz = 0.0;
        for (int c = 0; c < 8; ++c) {
          if (!cs[j].valid[c]) continue;
          const long kr_i = ((long)b * N + cs[j].row[c]) * C + head * d;
          const double* kr = k + kr_i;
          const double cq = dsq * cs[j].w[c], cv = pv * cs[j].w[c];
          for (int i = 0; i < d; ++i) {
            osum[i] += cq * kr[i];
            pdk[kr_i + i] += cq * qr[i];
            pdv[kr_i + i] += cv * dor[i];
          }
          const double gc = dsq * kdc[j * 8 + c] + pv * vdc[j * 8 + c];
          gx += cs[j].dwx[c] * gc;
          gy += cs[j].dwy[c] * gc;
          gz += cs[j].dwz[c] * gc;
        }
        gx *= clip_mult(pts[3 * j + 2], g->W);
        gy *= clip_mult(pts[3 * j + 1], g->H);
        gz *= clip_mult(pts[3 * j + 0], g->T);
        doffr[3 * j + 0] = g->T > 1 ? gx / (double)(g->T - 1) * g->offset_scale : 0.0;
        doffr[3 * j + 1] = g->H > 1 ? gy / (double)(g->H - 1) * g->offset_scale : 0.0;
        doffr[3 * j + 2] = g->W > 1 ? gz / (double)(g->W - 1) * g->offset_scale : 0.0;
      }
      for (int e = 0; e < G; ++e) {
        const double p = exp(s[K + e] - m) / l;
        const double kf = keep_factor(g, thr, b, t, h, w, head, K + e);
        const double dsq = p * (dpv[K + e] * kf - D) * g->softmax_scale;
        const double pv = p * kf;
        const long er = ((long)b * G + e) * C + head * d;
        for (int i = 0; i < d; ++i) {
          osum[i] += dsq * ek[er + i];
          pdek[er + i] += dsq * qr[i];
          pdev[er + i] += pv * dor[i];
        }
      }
      for (int i = 0; i < d; ++i) dq[qrow + i] = osum[i];
    }
#pragma omp critical
    {
      for (long i = 0; i < kvn; ++i) {
        dk[i] += pdk[i];
        dv[i] += pdv[i];
      }
      for (long i = 0; i < (G > 0 ? en : 0); ++i) {
        dek[i] += pdek[i];
        dev[i] += pdev[i];
      }
    }
    free(pdk); free(pdv); free(pdek); free(pdev); free(s); free(kdc); free(vdc); free(dpv);
    free(osum); free(cs); free(pts);
  }
}

/* Element i of a float32 (dtype 0) or bf16 (dtype 1, raw uint16 bits) array, as a double. */
static double load_el(const void* p, long i, int dtype) {
  if (dtype == 0) return (double)((const float*)p)[i];
  const uint32_t bits = (uint32_t)((const uint16_t*)p)[i] << 16;
  float f;
  memcpy(&f, &bits, sizeof f);
  return (double)f;
}

/* The core op (forward and backward, no extra keys) at a LIST of query rows of a large, possibly
 * time-sharded run, so that a run far too large for oracle_dsa_fwd / oracle_dsa_bwd can still be
 * checked row by row (attention.py:113-186; the same arithmetic as those two functions).
 *
 * The geometry names the GLOBAL volume.  The query rows of the run are frames
 * [q_frame0, q_frame0 + q_frames) of every sample; the K/V buffers hold frames
 * [kv_frame0, kv_frame0 + kv_frames).  qidx[i] = b * (q_frames*H*W) + local query row.
 * Per listed query i (all heads): q_rows / dout_rows [nq, >=C] (row stride row_ld), off_rows float32
 * [nq, nh*K*3] (the raw offsets, before offset_bias), bias float32 [nh*K*3] or NULL (added to the
 * offsets in one float32 rounding); k, v: the run's whole K/V buffers [B, kv_frames*H*W, >=C] (row
 * stride kv_ld).  Elements are float32 (dtype 0) or bf16 (dtype 1).
 * Outputs (double): out [nq, C], lse [nq, nh] (natural log), and when dout_rows is given dq [nq, C],
 * doff [nq, nh*K*3].  kv_slot (int32 [B*kv_rows], -1 = not watched; or NULL): dK / dV of the
 * listed queries are accumulated into dk_w / dv_w [nw, C] (overwritten) at the watched K/V rows.
 * Returns the number of sample corners that fell inside the volume but outside the K/V window
 * (those are skipped; a correct plan makes it 0). */
long oracle_dsa_rows(const oracle_geom* g, int q_frame0, int q_frames, int kv_frame0, int kv_frames, long nq,
                     const int64_t* qidx, const void* q_rows, const void* dout_rows, long row_ld,
                     const float* off_rows, const float* bias, const void* k, const void* v, long kv_ld, int dtype,
                     double* out, double* lse, double* dq, double* doff, const int32_t* kv_slot, long nw,
                     double* dk_w, double* dv_w) {
  const int K = g->kt * g->kh * g->kw, d = g->d, nh = g->nh;
  const long HW = (long)g->H * g->W, C = (long)nh * d, NQ = (long)q_frames * HW, NKV = (long)kv_frames * HW;
  const long nO = (long)nh * K * 3;
  const uint32_t thr = drop_threshold(g->dropout_p);
  const int want_bwd = dout_rows != NULL;
  long misses = 0;
  if (nw > 0) {
    memset(dk_w, 0, sizeof(double) * nw * C);
    memset(dv_w, 0, sizeof(double) * nw * C);
  }
#pragma omp parallel reduction(+ : misses)
  {
    double* s = (double*)malloc(sizeof(double) * K);
    double* kdc = (double*)malloc(sizeof(double) * K * 8);
    double* vdc = (double*)malloc(sizeof(double) * K * 8);
    double* dpv = (double*)malloc(sizeof(double) * K);
    double* qd = (double*)malloc(sizeof(double) * d);
    double* dod = (double*)malloc(sizeof(double) * d);
    double* acc = (double*)malloc(sizeof(double) * d);
    long* rows = (long*)malloc(sizeof(long) * K * 8);
    corner8* cs = (corner8*)malloc(sizeof(corner8) * K);
    float* pts = (float*)malloc(sizeof(float) * 3 * K);
    double* pdk = nw > 0 ? (double*)calloc(nw * C, sizeof(double)) : NULL;
    double* pdv = nw > 0 ? (double*)calloc(nw * C, sizeof(double)) : NULL;
#pragma omp for schedule(dynamic, 4)
    for (long item = 0; item < nq * nh; ++item) {
      const long i = item / nh;
      const int head = (int)(item % nh);
      const int b = (int)(qidx[i] / NQ);
      const long n = qidx[i] % NQ;
      const int t = q_frame0 + (int)(n / HW), h = (int)((n / g->W) % g->H), w = (int)(n % g->W);
      for (int c = 0; c < d; ++c) {
        qd[c] = load_el(q_rows, i * row_ld + head * d + c, dtype);
        dod[c] = want_bwd ? load_el(dout_rows, i * row_ld + head * d + c, dtype) : 0.0;
      }
      double m = -INFINITY;
      for (int j = 0; j < K; ++j) {
        float o3[3];
        for (int a = 0; a < 3; ++a) {
          const long ci = (long)head * K * 3 + 3 * j + a;
          o3[a] = bias ? off_rows[i * nO + ci] + bias[ci] : off_rows[i * nO + ci];
        }
        float pt, ph, pw;
        coords(g, t, h, w, j, o3, &pt, &ph, &pw);
        pts[3 * j] = pt; pts[3 * j + 1] = ph; pts[3 * j + 2] = pw;
        make_corners(g, pt, ph, pw, &cs[j]);
        double sj = 0.0, dpj = 0.0;
        for (int c = 0; c < 8; ++c) {
          double kd = 0.0, vd = 0.0;
          rows[j * 8 + c] = -1;
          if (cs[j].valid[c]) {
            const long tg = cs[j].row[c] / HW;
            if (tg < kv_frame0 || tg >= kv_frame0 + kv_frames) {
              if (cs[j].w[c] != 0.0) ++misses;
            } else {
              const long r = (long)b * NKV + cs[j].row[c] - (long)kv_frame0 * HW;
              rows[j * 8 + c] = r;
              for (int e = 0; e < d; ++e) {
                kd += qd[e] * load_el(k, r * kv_ld + head * d + e, dtype);
                if (want_bwd) vd += dod[e] * load_el(v, r * kv_ld + head * d + e, dtype);
              }
            }
          }
          kdc[j * 8 + c] = kd;
          vdc[j * 8 + c] = vd;
          sj += cs[j].w[c] * kd;
          dpj += cs[j].w[c] * vd;
        }
        s[j] = sj * g->softmax_scale;
        dpv[j] = dpj;
        if (s[j] > m) m = s[j];
      }
      double l = 0.0;
      for (int j = 0; j < K; ++j) l += exp(s[j] - m);
      lse[i * nh + head] = m + log(l);
      for (int e = 0; e < d; ++e) acc[e] = 0.0;
      for (int j = 0; j < K; ++j) {
        const double p = exp(s[j] - m) / l * keep_factor(g, thr, b, t, h, w, head, j);
        if (p == 0.0) continue;
        for (int c = 0; c < 8; ++c) {
          if (rows[j * 8 + c] < 0) continue;
          const double pw_ = p * cs[j].w[c];
          for (int e = 0; e < d; ++e) acc[e] += pw_ * load_el(v, rows[j * 8 + c] * kv_ld + head * d + e, dtype);
        }
      }
      for (int e = 0; e < d; ++e) out[i * C + head * d + e] = acc[e];
      if (!want_bwd) continue;
      double D = 0.0;
      for (int j = 0; j < K; ++j) D += exp(s[j] - m) / l * keep_factor(g, thr, b, t, h, w, head, j) * dpv[j];
      for (int e = 0; e < d; ++e) acc[e] = 0.0;
      for (int j = 0; j < K; ++j) {
        const double p = exp(s[j] - m) / l;
        const double kf = keep_factor(g, thr, b, t, h, w, head, j);
        const double dsq = p * (dpv[j] * kf - D) * g->softmax_scale;
        const double pv = p * kf;
        double gx = 0.0, gy = 0.0, gz = 0.0;
        for (int c = 0; c < 8; ++c) {
          const long r = rows[j * 8 + c];
          if (r < 0) continue;
          const double cq = dsq * cs[j].w[c], cv = pv * cs[j].w[c];
          const int slot = kv_slot ? kv_slot[r] : -1;
          for (int e = 0; e < d; ++e) acc[e] += cq * load_el(k, r * kv_ld + head * d + e, dtype);
          if (slot >= 0) {
            for (int e = 0; e < d; ++e) {
              pdk[(long)slot * C + head * d + e] += cq * qd[e];
              pdv[(long)slot * C + head * d + e] += cv * dod[e];
            }
          }
          const double gc = dsq * kdc[j * 8 + c] + pv * vdc[j * 8 + c];
          gx += cs[j].dwx[c] * gc;
          gy += cs[j].dwy[c] * gc;
          gz += cs[j].dwz[c] * gc;
        }
        gx *= clip_mult(pts[3 * j + 2], g->W);
        gy *= clip_mult(pts[3 * j + 1], g->H);
        gz *= clip_mult(pts[3 * j + 0], g->T);
        double* dr = doff + i * nO + (long)head * K * 3 + 3 * j;
        dr[0] = g->T > 1 ? gx / (double)(g->T - 1) * g->offset_scale : 0.0;
        dr[1] = g->H > 1 ? gy / (double)(g->H - 1) * g->offset_scale : 0.0;
        dr[2] = g->W > 1 ? gz / (double)(g->W - 1) * g->offset_scale : 0.0;
      }
      for (int e = 0; e < d; ++e) dq[i * C + head * d + e] = acc[e];
    }
    if (nw > 0) {
#pragma omp critical
      for (long e = 0; e < nw * C; ++e) {
        dk_w[e] += pdk[e];
        dv_w[e] += pdv[e];
      }
    }
    free(s); free(kdc); free(vdc); free(dpv); free(qd); free(dod); free(acc); free(rows); free(cs); free(pts);
    free(pdk); free(pdv);
  }
  return misses;
}

/* Depthwise 3D convolution, zero padding k//2, x/y [B, T*H*W, C], weight [kt*kh*kw, C]. */
void oracle_dwconv3d(int B, int T, int H, int W, int C, int kt, int kh, int kw, const double* x, const double* wt,
                     const double* bias, double* y) {
  const long N = (long)T * H * W;
#pragma omp parallel for schedule(static)
  for (long bn = 0; bn < (long)B * N; ++bn) {
    const int b = (int)(bn / N);
    const long n = bn % N;
    const int t = (int)(n / (H * W)), h = (int)((n / W) % H), w = (int)(n % W);
    double* yr = y + bn * C;
    for (int c = 0; c < C; ++c) yr[c] = bias ? bias[c] : 0.0;
    for (int it = 0; it < kt; ++it) {
      const int ti = t + it - kt / 2;
      if (ti < 0 || ti >= T) continue;
      for (int ih = 0; ih < kh; ++ih) {
        const int hi = h + ih - kh / 2;
        if (hi < 0 || hi >= H) continue;
        for (int iw = 0; iw < kw; ++iw) {
          const int wi = w + iw - kw / 2;
          if (wi < 0 || wi >= W) continue;
          const double* xr = x + ((long)b * N + ((long)ti * H + hi) * W + wi) * C;
          const double* wr = wt + (long)((it * kh + ih) * kw + iw) * C;
          for (int c = 0; c < C; ++c) yr[c] += wr[c] * xr[c];
        }
      }
    }
  }
}

/* Backward of oracle_dwconv3d: dx (overwritten), dw [K, C] and db [C] (overwritten). */
void oracle_dwconv3d_bwd(int B, int T, int H, int W, int C, int kt, int kh, int kw, const double* dy,
                         const double* x, const double* wt, double* dx, double* dw, double* db) {
  const long N = (long)T * H * W;
  const int K = kt * kh * kw;
#pragma omp parallel for schedule(static)
  for (long bn = 0; bn < (long)B * N; ++bn) {
    const int b = (int)(bn / N);
    const long n = bn % N;
    const int t = (int)(n / (H * W)), h = (int)((n / W) % H), w = (int)(n % W);
    double* xr = dx + bn * C;
    for (int c = 0; c < C; ++c) xr[c] = 0.0;
    for (int it = 0; it < kt; ++it) {
      const int to = t - it + kt / 2;
      if (to < 0 || to >= T) continue;
      for (int ih = 0; ih < kh; ++ih) {
        const int ho = h - ih + kh / 2;
        if (ho < 0 || ho >= H) continue;
        for (int iw = 0; iw < kw; ++iw) {
          const int wo = w - iw + kw / 2;
          if (wo < 0 || wo >= W) continue;
          const double* dr = dy + ((long)b * N + ((long)to * H + ho) * W + wo) * C;
          const double* wr = wt + (long)((it * kh + ih) * kw + iw) * C;
          for (int c = 0; c < C; ++c) xr[c] += wr[c] * dr[c];
        }
      }
    }
  }
#pragma omp parallel for schedule(static)
  for (int c = 0; c < C; ++c) {
    double sb = 0.0;
    for (long bn = 0; bn < (long)B * N; ++bn) sb += dy[bn * C + c];
    db[c] = sb;
    for (int tap = 0; tap < K; ++tap) {
      const int it = tap / (kh * kw), ih = (tap / kw) % kh, iw = tap % kw;
      double acc = 0.0;
      for (long bn = 0; bn < (long)B * N; ++bn) {
        const int b = (int)(bn / N);
        const long n = bn % N;
        const int t = (int)(n / (H * W)), h = (int)((n / W) % H), w = (int)(n % W);
        const int ti = t + it - kt / 2, hi = h + ih - kh / 2, wi = w + iw - kw / 2;
        if (ti < 0 || ti >= T || hi < 0 || hi >= H || wi < 0 || wi >= W) continue;
        acc += dy[bn * C + c] * x[((long)b * N + ((long)ti * H + hi) * W + wi) * C + c];
      }
      dw[(long)tap * C + c] = acc;
    }
  }
}

/* Exact (erf) GELU and its derivative, elementwise. */
void oracle_gelu(long n, const double* u, double* y) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; ++i) y[i] = 0.5 * u[i] * (1.0 + erf(u[i] * M_SQRT1_2));
}

void oracle_gelu_grad(long n, const double* u, double* gy) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; ++i) {
    const double cdf = 0.5 * (1.0 + erf(u[i] * M_SQRT1_2));
    const double pdf = exp(-0.5 * u[i] * u[i]) / sqrt(2.0 * M_PI);
    gy[i] = cdf + u[i] * pdf;
  }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
