/*
 * CPU restatement of the hot-path arithmetic - TEST INFRASTRUCTURE ONLY.
 *
 * Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as
 * the checker the CUDA kernels are compared against; never linked into or
 * called by the product (libspkv2_runtime.so).
 *
 * fp32 conv: the reference scalar conv (runtime/kernels/reference/conv/
 *   conv.c:3-62): per output, sum starts at the bias, accumulates x*w in
 *   (c, kh, kw) order, adds the residual (inputs[3]) and then applies the
 *   fused activation (kernel_common.c:100-108: 1 Relu, 2 x/(1+expf(-x))).
 * INT8 conv: the requantisation contract of the INT8 configs (the reference
 *   INT8 conv is ARM-dotprod only, conv_int8.c:13, and cannot run on x86):
 *     acc  = sum int32(w_q) * int32(x_q)           exact
 *     acc' = acc + b_q[c]
 *     v    = (float)acc' * M[c]                    one fp32 rounding
 *     v    = v + (float)r_q * R                    (residual) two roundings
 *     y_q  = clamp(rne(v), relu ? 0 : -128, 127)
 *   Built with -ffp-contract=off so no multiply-add is fused; the CUDA
 *   kernel uses __fmul_rn/__fadd_rn for the same reason.
 * fp32 conv with int8 output: y_q = clamp(rne(act(sum) * inv_sy), -128, 127).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>

static float act_f32(float v, int act) {
    if (act == 1) return v > 0.0f ? v : 0.0f;
    if (act == 2) return v / (1.0f + expf(-v));
    return v;
}

static int8_t sat_rne(float v, int lo) {
    float r = rintf(v); /* default rounding mode: nearest, ties to even */
    if (r < (float)lo) r = (float)lo;
    if (r > 127.0f) r = 127.0f;
    return (int8_t)r;
}

typedef struct {
    int N, C, H, W, M, KH, KW, OH, OW, sh, sw, ph, pw, dh, dw, group, act;
} ConvShape;

/* One fp32 output value following the reference loop order. */
static float conv_point_f32(const float *x, const float *w, const float *b, const ConvShape *s, int n, int m,
                            int oh, int ow) {
    const int Cg = s->C / s->group, Mg = s->M / s->group;
    const int g = m / Mg;
    float sum = b ? b[m] : 0.0f;
    for (int c = g * Cg; c < (g + 1) * Cg; c++) {
        const int wc = c - g * Cg;
        for (int kh = 0; kh < s->KH; kh++) {
            const int ih = oh * s->sh + kh * s->dh - s->ph;
            if (ih < 0 || ih >= s->H) continue;
            for (int kw = 0; kw < s->KW; kw++) {
                const int iw = ow * s->sw + kw * s->dw - s->pw;
                if (iw < 0 || iw >= s->W) continue;
                sum += x[(((size_t)n * s->C + c) * s->H + ih) * s->W + iw] *
                       w[(((size_t)m * Cg + wc) * s->KH + kh) * s->KW + kw];
            }
        }
    }
    return sum;
}

void oracle_conv2d_f32(const float *x, const float *w, const float *b, const float *res, float *y,
                       const ConvShape *s) {
    const long total = (long)s->N * s->M;
#pragma omp parallel for schedule(dynamic)
    for (long nm = 0; nm < total; nm++) {
        const int n = (int)(nm / s->M), m = (int)(nm % s->M);
        for (int oh = 0; oh < s->OH; oh++)
            for (int ow = 0; ow < s->OW; ow++) {
                const size_t yi = (((size_t)n * s->M + m) * s->OH + oh) * s->OW + ow;
                float v = conv_point_f32(x, w, b, s, n, m, oh, ow);
                if (res) v += res[yi];
                y[yi] = act_f32(v, s->act);
            }
    }
}

void oracle_conv2d_f32_to_i8(const float *x, const float *w, const float *b, int8_t *y, const ConvShape *s,
                             float inv_sy) {
    const long total = (long)s->N * s->M;
#pragma omp parallel for schedule(dynamic)
    for (long nm = 0; nm < total; nm++) {
        const int n = (int)(nm / s->M), m = (int)(nm % s->M);
        for (int oh = 0; oh < s->OH; oh++)
            for (int ow = 0; ow < s->OW; ow++) {
                const size_t yi = (((size_t)n * s->M + m) * s->OH + oh) * s->OW + ow;
                const float v = act_f32(conv_point_f32(x, w, b, s, n, m, oh, ow), s->act);
                y[yi] = sat_rne(v * inv_sy, -128);
            }
    }
}

/* INT8 conv.  acc_out (optional) receives the raw int32 accumulators
 * (without the bias) in NCHW order for bit-exact accumulator checks. */
void oracle_conv2d_i8(const int8_t *x, const int8_t *w, const int32_t *bq, const float *mscale, const int8_t *res,
                      float res_scale, int8_t *y, int32_t *acc_out, const ConvShape *s) {
    const int Cg = s->C / s->group, Mg = s->M / s->group;
    const int lo = s->act == 1 ? 0 : -128;
    const long total = (long)s->N * s->M;
#pragma omp parallel for schedule(dynamic)
    for (long nm = 0; nm < total; nm++) {
        const int n = (int)(nm / s->M), m = (int)(nm % s->M);
        const int g = m / Mg;
        for (int oh = 0; oh < s->OH; oh++)
            for (int ow = 0; ow < s->OW; ow++) {
                int32_t acc = 0;
                for (int c = g * Cg; c < (g + 1) * Cg; c++) {
                    const int wc = c - g * Cg;
                    for (int kh = 0; kh < s->KH; kh++) {
                        const int ih = oh * s->sh + kh * s->dh - s->ph;
                        if (ih < 0 || ih >= s->H) continue;
                        for (int kw = 0; kw < s->KW; kw++) {
                            const int iw = ow * s->sw + kw * s->dw - s->pw;
                            if (iw < 0 || iw >= s->W) continue;
                            acc += (int32_t)x[(((size_t)n * s->C + c) * s->H + ih) * s->W + iw] *
                                   (int32_t)w[(((size_t)m * Cg + wc) * s->KH + kh) * s->KW + kw];
                        }
                    }
                }
                const size_t yi = (((size_t)n * s->M + m) * s->OH + oh) * s->OW + ow;
                if (acc_out) acc_out[yi] = acc;
                const int32_t a = acc + (bq ? bq[m] : 0);
                float v = (float)a * mscale[m];
                if (res) {
                    const float r = (float)res[yi] * res_scale;
                    v = v + r;
                }
                y[yi] = sat_rne(v, lo);
            }
    }
}

/* Round-half-even saturation of one value, exported for known-answer tests. */
int oracle_sat_rne(float v, int lo) { return (int)sat_rne(v, lo); }

/* Weights-only INT8 conv (the reference compiler's own INT8 format; its
 * kernel is reference runtime/kernels/optimized/conv/conv_int8.c:86-119):
 * from the int32 accumulators of the int8 conv over the on-the-fly
 * quantised input, y = act(fmaf((float)acc, cs[m], b[m]) + res), cs[m] =
 * fp32(s_w[m] * s_x); the multiply-add fused as in the reference's vector
 * path, then the residual add and the activation (Relu, or SiLU with
 * expf).  NCHW order. */
void oracle_dequant_w8(const int32_t *acc, const float *cs, const float *b, const float *res, float *y,
                       const ConvShape *s) {
    const long spatial = (long)s->OH * s->OW;
    const long total = (long)s->N * s->M * spatial;
    for (long i = 0; i < total; i++) {
        const int m = (int)((i / spatial) % s->M);
        float v = fmaf((float)acc[i], cs[m], b ? b[m] : 0.0f);
        if (res) v = v + res[i];
        if (s->act == 1) v = v > 0.0f ? v : 0.0f;
        else if (s->act == 2) v = v / (1.0f + expf(-v));
        y[i] = v;
    }
}
