/*
 * sf_oracle.c -- TEST INFRASTRUCTURE ONLY. A plain-C CPU restatement of the
 * reference (hpcyhr/SparseFlow) algorithms on the spike-sparse conv path,
 * used as the checker in tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg. The product path never links or calls this file.
 *
 * Pinned against golden vectors produced by the reference itself
 * (tests/golden/make_golden.py; checked in tests/test_oracle_golden.py).
 *
 * Inputs arrive as float arrays. For the prescan, the caller has already
 * rounded x and the threshold to IEEE half (the reference prescans the fp16
 * cast of x and compares against the threshold in half), so the comparisons
 * here are exact.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static int imin(int a, int b) { return a < b ? a : b; }

/*
 * Receptive-field prescan. Follows Kernels/_prescan_common.py:32-189:
 *   group_max  = amax over the channels of each group of |x|     (:32-45)
 *   rf_max     = max_pool2d(group_max, k, s, p)                  (:169-177)
 *   tile_max   = max_pool2d(rf_max, (bh,bw), ceil_mode=True)     (:182-187)
 *   active     = tile_max > thr                                  (:188)
 * A max over a window holding a NaN is NaN (torch semantics), and NaN > thr
 * is false, so a NaN anywhere in a tile's receptive field clears that
 * group's bit. Classes: :57-70. Active ids: Kernels/conv2d.py:113-123.
 * layout 0 = NCHW, 1 = NHWC.
 */
int oracle_prescan2d(const float* x, int layout, int N, int C, int H, int W, int Ho, int Wo, int k, int s,
                     int p, int bh, int bw, int gs, float thr, int32_t* ag_mask, int32_t* tile_class,
                     int32_t* active_ids, int32_t* active_count) {
  const int G = (C + gs - 1) / gs;
  if (G > 32 || G <= 0) return 1;
  const int GH = (Ho + bh - 1) / bh, GW = (Wo + bw - 1) / bw;
  const uint32_t full = (G == 32) ? 0xffffffffu : ((1u << G) - 1u);
  uint32_t* act = (uint32_t*)calloc((size_t)H * W, sizeof(uint32_t));
  uint32_t* nanm = (uint32_t*)calloc((size_t)H * W, sizeof(uint32_t));
  if (!act || !nanm) {
    free(act);
    free(nanm);
    return 2;
  }
  int count = 0;
  for (int n = 0; n < N; ++n) {
    memset(act, 0, sizeof(uint32_t) * (size_t)H * W);
    memset(nanm, 0, sizeof(uint32_t) * (size_t)H * W);
    for (int c = 0; c < C; ++c) {
      const uint32_t bit = 1u << (c / gs);
      for (int ih = 0; ih < H; ++ih)
        for (int iw = 0; iw < W; ++iw) {
          const size_t idx = layout == 0 ? (((size_t)n * C + c) * H + ih) * W + iw
                                         : (((size_t)n * H + ih) * W + iw) * C + c;
          const float v = x[idx];
          if (isnan(v))
            nanm[ih * W + iw] |= bit;
          else if (fabsf(v) > thr)
            act[ih * W + iw] |= bit;
        }
    }
    for (int gh = 0; gh < GH; ++gh)
      for (int gw = 0; gw < GW; ++gw) {
        const int oh1 = imin((gh + 1) * bh, Ho), ow1 = imin((gw + 1) * bw, Wo);
        uint32_t a = 0, nn = 0;
        /* Union of the k x k windows of the tile's output pixels. */
        for (int oh = gh * bh; oh < oh1; ++oh)
          for (int ow = gw * bw; ow < ow1; ++ow)
            for (int dh = 0; dh < k; ++dh)
              for (int dw = 0; dw < k; ++dw) {
                const int ih = oh * s - p + dh, iw = ow * s - p + dw;
                if (ih < 0 || ih >= H || iw < 0 || iw >= W) continue;
                a |= act[ih * W + iw];
                nn |= nanm[ih * W + iw];
              }
        const uint32_t m = a & ~nn & full;
        const size_t t = ((size_t)n * GH + gh) * GW + gw;
        ag_mask[t] = (int32_t)m;
        tile_class[t] = m == 0 ? 0 : (m == full ? 2 : 1);
        if (m != 0 && active_ids) active_ids[count] = (int32_t)t;
        if (m != 0) ++count;
      }
  }
  if (active_count) *active_count = count;
  free(act);
  free(nanm);
  return 0;
}

/*
 * Direct conv2d, NCHW, square kernel, groups = 1, double accumulation (the
 * exact result the reference's CPU path, F.conv2d at Ops/sparse_conv2d.py:
 * 819-834, approximates in fp32). w: [Co][C][k][k]; bias may be NULL.
 */
void oracle_conv2d(const float* x, int N, int C, int H, int W, const float* w, const float* bias, int Co, int k,
                   int s, int p, float* y) {
  const int Ho = (H + 2 * p - k) / s + 1, Wo = (W + 2 * p - k) / s + 1;
  double* acc = (double*)malloc(sizeof(double) * (size_t)Ho * Wo);
  for (int n = 0; n < N; ++n)
    for (int co = 0; co < Co; ++co) {
      const double b = bias ? (double)bias[co] : 0.0;
      for (int i = 0; i < Ho * Wo; ++i) acc[i] = b;
      for (int c = 0; c < C; ++c) {
        const float* xc = x + ((size_t)n * C + c) * H * W;
        for (int ih = 0; ih < H; ++ih)
          for (int iw = 0; iw < W; ++iw) {
            const float v = xc[ih * W + iw];
            if (v == 0.0f) continue; /* exact: a zero contributes nothing */
            for (int dh = 0; dh < k; ++dh) {
              const int t = ih + p - dh;
              if (t < 0 || t % s) continue;
              const int oh = t / s;
              if (oh >= Ho) continue;
              for (int dw = 0; dw < k; ++dw) {
                const int u = iw + p - dw;
                if (u < 0 || u % s) continue;
                const int ow = u / s;
                if (ow >= Wo) continue;
                acc[oh * Wo + ow] += (double)v * (double)w[(((size_t)co * C + c) * k + dh) * k + dw];
              }
            }
          }
      }
      float* yo = y + ((size_t)n * Co + co) * Ho * Wo;
      for (int i = 0; i < Ho * Wo; ++i) yo[i] = (float)acc[i];
    }
  free(acc);
}

/*
 * One LIF step on a precomputed input current I (n elements); v in/out.
 * Rule of Ops/sparse_fused_conv_lif.py:283-292, evaluated in float with the
 * same operation order; v_reset is taken as 0 in the charge equation for the
 * soft reset (hard_reset == 0), as the reference does.
 */
void oracle_lif_step(const float* I, size_t n, float tau, float vth, float v_reset, int hard_reset,
                     int decay_input, float* v, float* spikes) {
  const float vr = hard_reset ? v_reset : 0.0f;
  for (size_t i = 0; i < n; ++i) {
    const float vp = v[i];
    float vt;
    if (decay_input)
      vt = vp + (I[i] - (vp - vr)) / tau;
    else
      vt = vp - (vp - vr) / tau + I[i];
    const int spike = vt >= vth;
    spikes[i] = spike ? 1.0f : 0.0f;
    v[i] = hard_reset ? (spike ? v_reset : vt) : (vt - (spike ? vth : 0.0f));
  }
}

/*
 * Multi-step conv + LIF. x: [T][N][C][H][W]; v: [N][Co][Ho][Wo] in/out;
 * spikes: [T][N][Co][Ho][Wo].
 */
void oracle_conv_lif(const float* x, int T, int N, int C, int H, int W, const float* w, const float* bias, int Co,
                     int k, int s, int p, float tau, float vth, float v_reset, int hard_reset, int decay_input,
                     float* v, float* spikes) {
  const int Ho = (H + 2 * p - k) / s + 1, Wo = (W + 2 * p - k) / s + 1;
  const size_t step_in = (size_t)N * C * H * W, step_out = (size_t)N * Co * Ho * Wo;
  float* cur = (float*)malloc(sizeof(float) * step_out);
  for (int t = 0; t < T; ++t) {
    oracle_conv2d(x + t * step_in, N, C, H, W, w, bias, Co, k, s, p, cur);
    oracle_lif_step(cur, step_out, tau, vth, v_reset, hard_reset, decay_input, v, spikes + t * step_out);
  }
  free(cur);
}
