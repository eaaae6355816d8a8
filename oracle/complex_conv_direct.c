/*
 * Plain C restatement of the complex Conv2d forward (cross-correlation with
 * zero padding), fp64 accumulation.
 *
 * TEST INFRASTRUCTURE ONLY: called from the oracle (tests, smoke, CPU
 * baseline) as the checker, never from the product path.
 *
 * Follows the four-real-Conv2d formula of the reference,
 * benchmarks/baseline.py:5-9:
 *     y_re = conv(x_re, w_re) - conv(x_im, w_im)
 *     y_im = conv(x_im, w_re) + conv(x_re, w_im)
 * with the output-size rule of csrc/complex_conv2d.cu:151-155 and the
 * cross-correlation mode of csrc/complex_conv2d.cu:194.
 *
 * Layouts: x planes NCHW, w planes KCRS, y planes NKPQ (all row-major).
 */
#include <stdint.h>

int ccv_oracle_direct_fprop(const double *x_re, const double *x_im,
                            const double *w_re, const double *w_im,
                            double *y_re, double *y_im,
                            int64_t n, int64_t h, int64_t w, int64_t c,
                            int64_t k, int64_t r, int64_t s,
                            int64_t stride_h, int64_t stride_w,
                            int64_t pad_h, int64_t pad_w) {
  if (n <= 0 || h <= 0 || w <= 0 || c <= 0 || k <= 0 || r <= 0 || s <= 0)
    return 1;
  if (stride_h <= 0 || stride_w <= 0 || pad_h < 0 || pad_w < 0) return 2;
  const int64_t p = (h + 2 * pad_h - r) / stride_h + 1;
  const int64_t q = (w + 2 * pad_w - s) / stride_w + 1;
  if (p <= 0 || q <= 0) return 3;

  for (int64_t in = 0; in < n; ++in) {
    for (int64_t ik = 0; ik < k; ++ik) {
      for (int64_t ip = 0; ip < p; ++ip) {
        for (int64_t iq = 0; iq < q; ++iq) {
          double acc_rr = 0.0, acc_ii = 0.0, acc_ir = 0.0, acc_ri = 0.0;
          for (int64_t ic = 0; ic < c; ++ic) {
            for (int64_t ir = 0; ir < r; ++ir) {
              const int64_t hh = ip * stride_h - pad_h + ir;
              if (hh < 0 || hh >= h) continue;
              for (int64_t is = 0; is < s; ++is) {
                const int64_t ww = iq * stride_w - pad_w + is;
                if (ww < 0 || ww >= w) continue;
                const int64_t xo = ((in * c + ic) * h + hh) * w + ww;
                const int64_t wo = ((ik * c + ic) * r + ir) * s + is;
                acc_rr += x_re[xo] * w_re[wo];  /* conv_real(x.real) */
                acc_ii += x_im[xo] * w_im[wo];  /* conv_imag(x.imag) */
                acc_ir += x_im[xo] * w_re[wo];  /* conv_real(x.imag) */
                acc_ri += x_re[xo] * w_im[wo];  /* conv_imag(x.real) */
              }
            }
          }
          const int64_t yo = ((in * k + ik) * p + ip) * q + iq;
          y_re[yo] = acc_rr - acc_ii;
          y_im[yo] = acc_ir + acc_ri;
        }
      }
    }
  }
  return 0;
}
