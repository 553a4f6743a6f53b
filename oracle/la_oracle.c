/*
 * Double-precision C restatement of the UPLiFT Local Attender --
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Follows the reference's non-fast LocalAttender.forward
 * (uplift/uplift.py:801-847): 1x1 projection conv1 with bias (:810),
 * residual_auto truncation / zero padding (:26-39, :811-812), replicate
 * padding by pn and the K shifted views (:784-798), softmax over K (:828),
 * child mapping [B, K, H, I, W, I] (:829-830) and the sum over K (:835-837).
 * hardmax = one-hot of the first argmax as in the Triton module's fallback
 * (uplift/kernels/triton_attender.py:421-424).
 *
 * All inputs are fp32 NCHW contiguous; every sum is accumulated in double.
 * Build: `make -C oracle` (gcc; OpenMP over batch x output rows when
 * built with -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* guide [B][Cg][Ho][Wo], value [B][C][H][W], weight [K][Cg], bias [K] or
 * NULL, offsets [K][2] (dy, dx), out [B][C][Ho][Wo] with Ho = I*H, Wo = I*W.
 * If logits != NULL it is read as [B][K][Ho][Wo] and guide/weight/bias are
 * ignored (the pre-projected-logit entry point).  Returns 0 on success. */
int la_oracle_forward(const float* guide, const float* value, const float* weight,
                      const float* bias, const float* logits, float* out,
                      int B, int Cg, int C, int H, int W, int I, int K,
                      const int8_t* offsets, int conv_res, int hardmax) {
  if (K < 1 || K > 64 || I < 1) return 1;
  const int Ho = I * H, Wo = I * W;
  const long long gplane = (long long)Ho * Wo;
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < B; ++b) {
    for (int y = 0; y < Ho; ++y) {
      double lg[64], p[64];
      for (int x = 0; x < Wo; ++x) {
        const long long pix = (long long)y * Wo + x;
        for (int k = 0; k < K; ++k) {
          double s;
          if (logits) {
            s = logits[((long long)b * K + k) * gplane + pix];
          } else {
            s = bias ? bias[k] : 0.0;
            for (int c = 0; c < Cg; ++c)
              s += (double)weight[(long long)k * Cg + c] * guide[((long long)b * Cg + c) * gplane + pix];
            if (conv_res && k < Cg) s += guide[((long long)b * Cg + k) * gplane + pix];
          }
          lg[k] = s;
        }
        if (hardmax) {
          int best = 0;
          for (int k = 1; k < K; ++k)
            if (lg[k] > lg[best]) best = k;
          for (int k = 0; k < K; ++k) p[k] = (k == best) ? 1.0 : 0.0;
        } else {
          double m = lg[0], z = 0.0;
          for (int k = 1; k < K; ++k) m = lg[k] > m ? lg[k] : m;
          for (int k = 0; k < K; ++k) { p[k] = exp(lg[k] - m); z += p[k]; }
          for (int k = 0; k < K; ++k) p[k] /= z;
        }
        const int h = y / I, w = x / I;
        for (int c = 0; c < C; ++c) {
          const float* vp = value + ((long long)b * C + c) * H * W;
          double acc = 0.0;
          for (int k = 0; k < K; ++k) {
            const int ny = clampi(h + offsets[2 * k], 0, H - 1);
            const int nx = clampi(w + offsets[2 * k + 1], 0, W - 1);
            acc += p[k] * vp[(long long)ny * W + nx];
          }
          out[((long long)b * C + c) * gplane + pix] = (float)acc;
        }
      }
    }
  }
  return 0;
}
