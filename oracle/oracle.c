/*
 * TEST INFRASTRUCTURE ONLY -- the CPU restatement ("port") of the reference's
 * lowered-op loop nests that the B200 kernels are checked against.  Nothing in
 * the product links this file; tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load it through oracle/oracle.py.
 *
 * Every function restates the arithmetic of one reference C template, in the
 * same statement order and with the same C types, so that gcc produces the
 * same bits as the reference's generated C (pinned by the golden fixtures in
 * tests/golden/, which come from the reference's own generated C).  Build
 * with the flags the reference's generated C is built with: -std=c99 -O2, no
 * -march, no -ffast-math (x86-64 baseline SSE2: no FMA contraction, float
 * arithmetic rounded per operation, _Float16 arithmetic evaluated in float and
 * rounded to half on assignment).
 *
 * Citations are paths inside the reference project
 * (src/emx_onnx_cgen/templates/... and src/emx_onnx_cgen/ir/ops/...).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>

typedef _Float16 f16;

/* The reference routes fp16 transcendental/min-max calls through helpers whose
 * parameters are _Float16, so the argument is rounded to half before the
 * double libm call (shared/scalar_functions.py:503-506). */
static inline f16 f16_exp(f16 a) { return exp(a); }
static inline f16 f16_max(f16 a, f16 b) { return fmax(a, b); }

/* ---------------------------------------------------------------------------
 * QLinearConv, 2-D, NCHW / OIHW.  templates/qlinear_conv_op.c.j2:1-45,
 * ir/ops/nn.py:4875-4951 (float compute type; nearbyint evaluated in double).
 * x_signed / w_signed / y_signed select int8 vs uint8 storage.
 * ------------------------------------------------------------------------- */
void orc_qlinear_conv2d(const void *x_, int x_signed, int n_batch, int c_in, int h_in, int w_in,
                        float x_scale, int x_zero,
                        const void *w_, int w_signed, int c_out, int k_h, int k_w,
                        const float *w_scale, int w_scale_per_channel,
                        const int32_t *w_zero, int w_zero_per_channel,
                        float y_scale, int y_zero,
                        const int32_t *bias,
                        int stride_h, int stride_w, int pad_top, int pad_left,
                        int dil_h, int dil_w, int group,
                        void *y_, int y_signed, int h_out, int w_out)
{
    const uint8_t *xu = (const uint8_t *)x_;
    const int8_t *xs = (const int8_t *)x_;
    const uint8_t *wu = (const uint8_t *)w_;
    const int8_t *ws = (const int8_t *)w_;
    uint8_t *yu = (uint8_t *)y_;
    int8_t *ys = (int8_t *)y_;
    const int gic = c_in / group, goc = c_out / group;
    const float ymin = y_signed ? -128.0f : 0.0f;
    const float ymax = y_signed ? 127.0f : 255.0f;
    for (int n = 0; n < n_batch; ++n) {
        for (int g = 0; g < group; ++g) {
            for (int oc = 0; oc < goc; ++oc) {
                const int ocg = g * goc + oc;
                const float scale = ((float)x_scale) *
                                    ((float)w_scale[w_scale_per_channel ? ocg : 0]) /
                                    ((float)y_scale);
                const int32_t wz = w_zero ? w_zero[w_zero_per_channel ? ocg : 0] : 0;
                for (int oh = 0; oh < h_out; ++oh) {
                    for (int ow = 0; ow < w_out; ++ow) {
                        int32_t acc = 0;
                        if (bias) acc += bias[ocg];
                        for (int ic = 0; ic < gic; ++ic) {
                            const int icg = g * gic + ic;
                            for (int kh = 0; kh < k_h; ++kh) {
                                for (int kw = 0; kw < k_w; ++kw) {
                                    const int ih = oh * stride_h + kh * dil_h - pad_top;
                                    const int iw = ow * stride_w + kw * dil_w - pad_left;
                                    if (ih >= 0 && ih < h_in && iw >= 0 && iw < w_in) {
                                        const size_t xi = (((size_t)n * c_in + icg) * h_in + ih) * w_in + iw;
                                        const size_t wi = (((size_t)ocg * gic + ic) * k_h + kh) * k_w + kw;
                                        const int32_t xv = (x_signed ? (int32_t)xs[xi] : (int32_t)xu[xi]) - (int32_t)x_zero;
                                        const int32_t wv = (w_signed ? (int32_t)ws[wi] : (int32_t)wu[wi]) - wz;
                                        acc += xv * wv;
                                    }
                                }
                            }
                        }
                        float scaled = ((float)acc) * scale;
                        float rounded = nearbyint((double)scaled) + (float)y_zero;
                        rounded = fmaxf(rounded, ymin);
                        rounded = fminf(rounded, ymax);
                        const size_t yi = (((size_t)n * c_out + ocg) * h_out + oh) * w_out + ow;
                        if (y_signed) ys[yi] = (int8_t)rounded; else yu[yi] = (uint8_t)rounded;
                    }
                }
            }
        }
    }
}

/* ---------------------------------------------------------------------------
 * com.microsoft QLinearAdd, same-shape operands.
 * templates/qlinear_add_op.c.j2:1-21 (float compute type, nearbyintf).
 * ------------------------------------------------------------------------- */
void orc_qlinear_add(const void *a_, int a_signed, float a_scale, int a_zero,
                     const void *b_, int b_signed, float b_scale, int b_zero,
                     float y_scale, int y_zero, void *y_, int y_signed, size_t count)
{
    const float a_s = (float)a_scale, b_s = (float)b_scale, y_s = (float)y_scale;
    const int32_t az = a_zero, bz = b_zero;
    const float yz = (float)y_zero;
    const float ymin = y_signed ? -128.0f : 0.0f, ymax = y_signed ? 127.0f : 255.0f;
    for (size_t i = 0; i < count; ++i) {
        const int32_t av = a_signed ? (int32_t)((const int8_t *)a_)[i] : (int32_t)((const uint8_t *)a_)[i];
        const int32_t bv = b_signed ? (int32_t)((const int8_t *)b_)[i] : (int32_t)((const uint8_t *)b_)[i];
        float a_real = ((float)(av - az)) * a_s;
        float b_real = ((float)(bv - bz)) * b_s;
        float scaled = (a_real + b_real) / y_s + yz;
        float rounded = nearbyintf(scaled);
        rounded = fmaxf(rounded, ymin);
        rounded = fminf(rounded, ymax);
        if (y_signed) ((int8_t *)y_)[i] = (int8_t)rounded; else ((uint8_t *)y_)[i] = (uint8_t)rounded;
    }
}

/* ---------------------------------------------------------------------------
 * Gemm fp32 (float accumulator, "simple" strategy).  templates/gemm_op.c.j2:1-40.
 * bias_mode: 0 none, 1 scalar, 2 per column j ([N]), 3 per row i ([M]), 4 full [M,N].
 * ------------------------------------------------------------------------- */
void orc_gemm_f32(const float *a, const float *b, const float *c, int bias_mode,
                  int m, int n, int k, int trans_a, int trans_b,
                  float alpha, float beta, float *y)
{
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            float acc = 0.0f;
            for (int kk = 0; kk < k; ++kk) {
                const float a_val = trans_a ? a[(size_t)kk * m + i] : a[(size_t)i * k + kk];
                const float b_val = trans_b ? b[(size_t)j * k + kk] : b[(size_t)kk * n + j];
                acc += a_val * b_val;
            }
            if (bias_mode) {
                float bias;
                switch (bias_mode) {
                case 1: bias = c[0]; break;
                case 2: bias = c[j]; break;
                case 3: bias = c[i]; break;
                default: bias = c[(size_t)i * n + j]; break;
                }
                y[(size_t)i * n + j] = acc * alpha + bias * beta;
            } else {
                y[(size_t)i * n + j] = acc * alpha;
            }
        }
    }
}

/* Relu: ref_scalar_f32_relu = a > 0.0f ? a : 0.0f (shared/scalar_functions.py RELU). */
void orc_relu_f32(const float *x, float *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* ---------------------------------------------------------------------------
 * com.microsoft MatMulNBits, bits=4, accuracy_level 0, fp16 A, float accumulator.
 * templates/matmul_nbits_op.c.j2:1-58; B packed [N][n_blocks][block/2], low
 * nibble first.  Zero points (ir/ops/nn.py:1172, lowering/matmul_nbits.py:
 * 171-185): absent -> 8; uint8 of rank >= 2 -> packed 4-bit per block, block
 * b in byte b/2 at shift (b*4)%8; rank 1 -> one per column (low nibble).
 * Scales [N][n_blocks] (per block) or [N].  Bias [N] (fp16) is added to the
 * float accumulator after the k loop; the result is cast to _Float16.
 * ------------------------------------------------------------------------- */
void orc_matmul_nbits_f16(const f16 *a, const uint8_t *b, const f16 *scales, int scales_per_block,
                          const uint8_t *zero_points, int zp_per_block, const f16 *bias,
                          int m, int n, int k, int block, f16 *y)
{
    const int n_blocks = (k + block - 1) / block;
    const int blob = block / 2;
    const int zp_cols = (n_blocks * 4 + 7) / 8;
    for (int i0 = 0; i0 < m; ++i0) {
        for (int i1 = 0; i1 < n; ++i1) {
            float acc = 0.0f;
            for (int kk = 0; kk < k; ++kk) {
                const int block_idx = kk / block;
                const int k_in_block = kk % block;
                const int byte_idx = k_in_block * 4 / 8;
                const int bit_shift = (k_in_block * 4) % 8;
                const int quant_val = ((int)(unsigned char)b[((size_t)i1 * n_blocks + block_idx) * blob + byte_idx] >> bit_shift) & 15;
                int zp = 8;
                if (zero_points && zp_per_block)
                    zp = ((int)zero_points[(size_t)i1 * zp_cols + block_idx * 4 / 8] >> ((block_idx * 4) % 8)) & 15;
                else if (zero_points)
                    zp = (int)zero_points[i1] & 15;
                const float s = (float)scales[scales_per_block ? (size_t)i1 * n_blocks + block_idx : (size_t)i1];
                const float dequant = ((float)quant_val - (float)zp) * s;
                acc += (float)a[(size_t)i0 * k + kk] * dequant;
            }
            if (bias) acc += (float)bias[i1];
            y[(size_t)i0 * n + i1] = (f16)acc;
        }
    }
}

/* ---------------------------------------------------------------------------
 * com.microsoft MatMulNBits, bits=4, accuracy_level 4 on fp16 A: the int8
 * activation path (templates/matmul_nbits_int8_op.c.j2:1-78, selected at
 * ir/ops/nn.py:1183-1190).  Per row and K block: amax = max |a| (float),
 * a_scale = amax / 127, a_inv = amax > 0 ? 127 / amax : 0, qa = int8 of
 * nearbyintf(a * a_inv) clamped to [-128, 127]; per output: acc = 0, then per
 * block in order acc += (float)isum * (a_scale * b_scale), isum the exact
 * int32 sum of qa * (q - zp) over the block (a partial last block stops at K);
 * bias added after the blocks, result cast to _Float16.  Weight, scale and
 * zero-point layouts as in orc_matmul_nbits_f16.
 * ------------------------------------------------------------------------- */
void orc_matmul_nbits_i8_f16(const f16 *a, const uint8_t *b, const f16 *scales, int scales_per_block,
                             const uint8_t *zero_points, int zp_per_block, const f16 *bias,
                             int m, int n, int k, int block, f16 *y)
{
    const int n_blocks = (k + block - 1) / block;
    const int blob = block / 2;
    const int zp_cols = (n_blocks * 4 + 7) / 8;
    int8_t *qa = (int8_t *)malloc((size_t)(k > 0 ? k : 1));
    float *a_scale = (float *)malloc(sizeof(float) * (size_t)(n_blocks > 0 ? n_blocks : 1));
    for (int i0 = 0; i0 < m; ++i0) {
        const f16 *arow = a + (size_t)i0 * k;
        for (int blk = 0; blk < n_blocks; ++blk) {
            float amax = 0.0f;
            for (int kk = 0; kk < block; ++kk) {
                const int kx = blk * block + kk;
                if (kx >= k) break;
                const float av = fabsf((float)arow[kx]);
                if (av > amax) amax = av;
            }
            a_scale[blk] = amax / (float)127;
            const float a_inv = amax > 0.0f ? (float)127 / amax : 0.0f;
            for (int kk = 0; kk < block; ++kk) {
                const int kx = blk * block + kk;
                if (kx >= k) break;
                float q = nearbyintf((float)arow[kx] * a_inv);
                if (q > (float)127) q = (float)127;
                if (q < (float)-128) q = (float)-128;
                qa[kx] = (int8_t)q;
            }
        }
        for (int i1 = 0; i1 < n; ++i1) {
            float acc = 0.0f;
            for (int blk = 0; blk < n_blocks; ++blk) {
                int32_t isum = 0;
                for (int kk = 0; kk < block; ++kk) {
                    const int kx = blk * block + kk;
                    if (kx >= k) break;
                    const int quant_val = ((int)(unsigned char)b[((size_t)i1 * n_blocks + blk) * blob + kk * 4 / 8]
                                           >> ((kk * 4) % 8)) & 15;
                    int zp = 8;
                    if (zero_points && zp_per_block)
                        zp = ((int)zero_points[(size_t)i1 * zp_cols + blk * 4 / 8] >> ((blk * 4) % 8)) & 15;
                    else if (zero_points)
                        zp = (int)zero_points[i1] & 15;
                    isum += (int32_t)qa[kx] * (int32_t)(quant_val - zp);
                }
                const float b_scale = (float)scales[scales_per_block ? (size_t)i1 * n_blocks + blk : (size_t)i1];
                acc += (float)isum * (a_scale[blk] * b_scale);
            }
            if (bias) acc += (float)bias[i1];
            y[(size_t)i0 * n + i1] = (f16)acc;
        }
    }
    free(qa);
    free(a_scale);
}

/* Swish fp16: a / (1.0 + exp(-alpha * a)) with a double-precision exp
 * (shared/scalar_functions.py:880-896; double libm call for f16, :503-506). */
void orc_swish_f16(const f16 *x, f16 *y, size_t count, float alpha_f)
{
    const f16 alpha = (f16)alpha_f;
    for (size_t i = 0; i < count; ++i) {
        const f16 a = x[i];
        y[i] = a / (1.0 + exp(-alpha * a));
    }
}

/* Sigmoid fp16: 1.0 / (1.0 + exp(-a)) in double (shared/scalar_functions.py:727-731). */
void orc_sigmoid_f16(const f16 *x, f16 *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) {
        const f16 a = x[i];
        y[i] = 1.0 / (1.0 + exp(-a));
    }
}

/* Mul fp16 (binary_op.c.j2 with ref_scalar_f16_mul = a * b). */
void orc_mul_f16(const f16 *a, const f16 *b, f16 *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) {
        const f16 av = a[i], bv = b[i];
        y[i] = av * bv;
    }
}

/* Mul / Add fp32 */
void orc_mul_f32(const float *a, const float *b, float *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) y[i] = a[i] * b[i];
}

void orc_add_f32(const float *a, const float *b, float *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) y[i] = a[i] + b[i];
}

/* Sigmoid / Tanh fp32 (ref_scalar_f32_sigmoid = 1.0f / (1.0f + expf(-a)); tanhf). */
void orc_sigmoid_f32(const float *x, float *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) y[i] = 1.0f / (1.0f + expf(-x[i]));
}

void orc_tanh_f32(const float *x, float *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) y[i] = tanhf(x[i]);
}

/* ---------------------------------------------------------------------------
 * Attention (opset 23), fp16, 4-D [batch, heads, seq, head] layout, no mask
 * input, no past/present, softcap 0.  templates/attention_op.c.j2:1-189 in the
 * fp16 instantiation: scores, softmax sum and P.V accumulate in _Float16; exp
 * is the double libm exp (ref_scalar_f16_exp).  kv_heads may divide q_heads.
 * ------------------------------------------------------------------------- */
void orc_attention_f16(const f16 *q, const f16 *k, const f16 *v, f16 *out,
                       int batch, int q_heads, int kv_heads, int q_seq, int kv_seq,
                       int head_dim, int v_head_dim, float scale_f, int is_causal)
{
    const f16 scale = (f16)scale_f;
    const int group = q_heads / kv_heads;
    f16 *scores = (f16 *)malloc(sizeof(f16) * (size_t)kv_seq);
    f16 *weights = (f16 *)malloc(sizeof(f16) * (size_t)kv_seq);
    const int past = kv_seq - q_seq;
    for (int b = 0; b < batch; ++b) {
        for (int h = 0; h < q_heads; ++h) {
            const int kvh = h / group;
            const f16 *qb = q + (((size_t)b * q_heads + h) * q_seq) * head_dim;
            const f16 *kb = k + (((size_t)b * kv_heads + kvh) * kv_seq) * head_dim;
            const f16 *vb = v + (((size_t)b * kv_heads + kvh) * kv_seq) * v_head_dim;
            f16 *ob = out + (((size_t)b * q_heads + h) * q_seq) * v_head_dim;
            for (int qi = 0; qi < q_seq; ++qi) {
                f16 max_score = -INFINITY;
                for (int ki = 0; ki < kv_seq; ++ki) {
                    f16 score = 0.0f;
                    for (int d = 0; d < head_dim; ++d) {
                        f16 q_val = qb[(size_t)qi * head_dim + d];
                        f16 k_val = kb[(size_t)ki * head_dim + d];
                        score += q_val * k_val;
                    }
                    score *= scale;
                    f16 bias = 0.0f;
                    if (is_causal && ki > qi + past) bias = -INFINITY;
                    f16 score_bias = score + bias;
                    scores[ki] = score_bias;
                    max_score = f16_max(max_score, score_bias);
                }
                f16 sum = 0.0f;
                for (int ki = 0; ki < kv_seq; ++ki) {
                    f16 weight = 0.0f;
                    if (max_score != -INFINITY) weight = f16_exp(scores[ki] - max_score);
                    weights[ki] = weight;
                    sum += weight;
                }
                f16 inv_sum = sum == 0.0f ? 0.0f : (f16)(f16)1.0f / sum;
                for (int vd = 0; vd < v_head_dim; ++vd) {
                    f16 acc = 0.0f;
                    for (int ki = 0; ki < kv_seq; ++ki) {
                        f16 weight = weights[ki] * inv_sum;
                        acc += weight * vb[(size_t)ki * v_head_dim + vd];
                    }
                    ob[(size_t)qi * v_head_dim + vd] = acc;
                }
            }
        }
    }
    free(scores);
    free(weights);
}

/* ---------------------------------------------------------------------------
 * LSTM fp32, forward direction, layout 0, zero initial state, activations
 * Sigmoid/Tanh/Tanh, gate order i,o,f,c, bias = Wb + Rb added after the dot
 * products.  templates/lstm_op.c.j2:1-175.  bias may be NULL.
 * ------------------------------------------------------------------------- */
void orc_lstm_f32(const float *x, const float *w, const float *r, const float *bias,
                  int seq, int batch, int input, int hidden,
                  float *y, float *y_h, float *y_c)
{
    float *h_prev = (float *)calloc((size_t)batch * hidden, sizeof(float));
    float *c_prev = (float *)calloc((size_t)batch * hidden, sizeof(float));
    float *h_next = (float *)malloc(sizeof(float) * (size_t)hidden);
    float *c_next = (float *)malloc(sizeof(float) * (size_t)hidden);
    const int H = hidden;
    for (int b = 0; b < batch; ++b) {
        for (int step = 0; step < seq; ++step) {
            const int t = step;
            for (int h = 0; h < H; ++h) {
                float gate_i = 0.0f, gate_o = 0.0f, gate_f = 0.0f, gate_c = 0.0f;
                for (int i = 0; i < input; ++i) {
                    const float x_val = x[((size_t)t * batch + b) * input + i];
                    gate_i += x_val * w[(size_t)h * input + i];
                    gate_o += x_val * w[(size_t)(H + h) * input + i];
                    gate_f += x_val * w[(size_t)(2 * H + h) * input + i];
                    gate_c += x_val * w[(size_t)(3 * H + h) * input + i];
                }
                for (int i = 0; i < H; ++i) {
                    const float h_val = h_prev[(size_t)b * H + i];
                    gate_i += h_val * r[(size_t)h * H + i];
                    gate_o += h_val * r[(size_t)(H + h) * H + i];
                    gate_f += h_val * r[(size_t)(2 * H + h) * H + i];
                    gate_c += h_val * r[(size_t)(3 * H + h) * H + i];
                }
                if (bias) {
                    gate_i += bias[h] + bias[4 * H + h];
                    gate_o += bias[H + h] + bias[5 * H + h];
                    gate_f += bias[2 * H + h] + bias[6 * H + h];
                    gate_c += bias[3 * H + h] + bias[7 * H + h];
                }
                const float i_gate = 1.0f / (1.0f + expf(-gate_i));
                const float f_gate = 1.0f / (1.0f + expf(-gate_f));
                const float c_gate = tanhf(gate_c);
                const float c_new = f_gate * c_prev[(size_t)b * H + h] + i_gate * c_gate;
                const float o_gate = 1.0f / (1.0f + expf(-gate_o));
                const float h_new = o_gate * tanhf(c_new);
                c_next[h] = c_new;
                h_next[h] = h_new;
                y[((size_t)step * batch + b) * H + h] = h_new;
            }
            for (int h = 0; h < H; ++h) {
                c_prev[(size_t)b * H + h] = c_next[h];
                h_prev[(size_t)b * H + h] = h_next[h];
            }
        }
    }
    memcpy(y_h, h_prev, sizeof(float) * (size_t)batch * H);
    memcpy(y_c, c_prev, sizeof(float) * (size_t)batch * H);
    free(h_prev); free(c_prev); free(h_next); free(c_next);
}

/* ---------------------------------------------------------------------------
 * QLinearMatMul, 2-D B, per-tensor parameters, f32 scales (ir/ops/nn.py:
 * 710-769, templates/qlinear_matmul_op.c.j2:1-81): int32 accumulation of
 * (a - za) * (b - zb); if the double multiplier s_a*s_b/s_y is representable
 * in 31 fractional bits (within 1e-12) the integer path rounds
 * acc*multiplier >> frac_bits half-to-even, else (double)acc * (double)scale
 * + zy is rounded by llrint, scale being the float expression s_a*s_b/s_y.
 * ------------------------------------------------------------------------- */
void orc_qlinear_matmul(const uint8_t *a, int a_signed, const uint8_t *b, int b_signed, float sa, int za,
                        float sb, int zb, float sy, int zy, int y_signed, int m, int k, int n, uint8_t *y)
{
    const float scale = ((float)sa) * ((float)sb) / ((float)sy);
    const double real_multiplier = ((double)sa) * ((double)sb) / ((double)sy);
    int frac_bits = 31;
    double scaled_multiplier = ldexp(real_multiplier, frac_bits);
    while (frac_bits > 0 && fabs(scaled_multiplier) > (double)INT32_MAX) {
        --frac_bits;
        scaled_multiplier = ldexp(real_multiplier, frac_bits);
    }
    const int64_t mult = (int64_t)llround(scaled_multiplier);
    const double rq_scale = ldexp((double)mult, -frac_bits);
    const double err = fabs(real_multiplier - rq_scale);
    const double tol = fmax(1e-12, fabs(real_multiplier) * 1e-12);
    const int use_int = isfinite(real_multiplier) && err <= tol;
    const uint64_t mask = frac_bits > 0 ? (((uint64_t)1u << frac_bits) - 1u) : 0u;
    const uint64_t half = frac_bits > 0 ? ((uint64_t)1u << (frac_bits - 1)) : 0u;
    const int64_t lo = y_signed ? -128 : 0, hi = y_signed ? 127 : 255;
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            int32_t acc = 0;
            for (int kk = 0; kk < k; ++kk) {
                const int32_t av = a_signed ? (int32_t)(int8_t)a[(size_t)i * k + kk] : (int32_t)a[(size_t)i * k + kk];
                const int32_t bv = b_signed ? (int32_t)(int8_t)b[(size_t)kk * n + j] : (int32_t)b[(size_t)kk * n + j];
                acc += (av - za) * (bv - zb);
            }
            int64_t q;
            if (use_int) {
                int64_t r = (int64_t)acc * mult;
                if (frac_bits > 0) {
                    uint64_t mag = r < 0 ? (uint64_t)(-r) : (uint64_t)r;
                    uint64_t quo = mag >> frac_bits, rem = mag & mask;
                    if (rem > half || (rem == half && (quo & 1u))) ++quo;
                    r = r < 0 ? -(int64_t)quo : (int64_t)quo;
                }
                q = r + (int64_t)zy;
            } else {
                const double scaled = ((double)acc) * (double)scale + (double)zy;
                q = (int64_t)llrint(scaled);
            }
            if (q < lo) q = lo; else if (q > hi) q = hi;
            y[(size_t)i * n + j] = (uint8_t)(int8_t)q;
        }
    }
}

/* MatMulInteger (templates/matmul_integer_op.c.j2): int32 sum of (a - za) * (b - zb). */
void orc_matmul_integer(const uint8_t *a, int a_signed, const uint8_t *b, int b_signed, int za, int zb,
                        int m, int k, int n, int32_t *y)
{
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            int32_t acc = 0;
            for (int kk = 0; kk < k; ++kk) {
                const int32_t av = a_signed ? (int32_t)(int8_t)a[(size_t)i * k + kk] : (int32_t)a[(size_t)i * k + kk];
                const int32_t bv = b_signed ? (int32_t)(int8_t)b[(size_t)kk * n + j] : (int32_t)b[(size_t)kk * n + j];
                acc += (av - za) * (bv - zb);
            }
            y[(size_t)i * n + j] = acc;
        }
}

/* Conv fp32, 2-D (templates/conv_op.c.j2): acc = bias (or 0); in-bounds taps
 * in (ic, kh, kw) order: acc += x * w. */
void orc_conv2d_f32(const float *x, const float *w, const float *bias, int n, int c, int h, int wd, int oc,
                    int kh, int kw, int sh, int sw, int pt, int pl, int dh, int dw, int group, int oh, int ow,
                    float *y)
{
    const int gic = c / group, goc = oc / group;
    for (int b = 0; b < n; ++b)
        for (int g = 0; g < group; ++g)
            for (int o = 0; o < goc; ++o) {
                const int og = g * goc + o;
                for (int yy = 0; yy < oh; ++yy)
                    for (int xx = 0; xx < ow; ++xx) {
                        float acc = bias ? bias[og] : 0.0f;
                        for (int ic = 0; ic < gic; ++ic) {
                            const int icg = g * gic + ic;
                            for (int a = 0; a < kh; ++a)
                                for (int bb = 0; bb < kw; ++bb) {
                                    const int iy = yy * sh + a * dh - pt, ix = xx * sw + bb * dw - pl;
                                    if (iy >= 0 && iy < h && ix >= 0 && ix < wd)
                                        acc += x[(((size_t)b * c + icg) * h + iy) * wd + ix] *
                                               w[(((size_t)og * gic + ic) * kh + a) * kw + bb];
                                }
                        }
                        y[(((size_t)b * oc + og) * oh + yy) * ow + xx] = acc;
                    }
            }
}

/* Softmax fp32 over one axis (templates/softmax_op.c.j2): fmaxf chain, expf,
 * sequential float sum, division. */
void orc_softmax_f32(const float *x, float *y, long outer, long axis, long inner)
{
    for (long o = 0; o < outer; ++o)
        for (long i = 0; i < inner; ++i) {
            const long base = o * axis * inner + i;
            float mx = x[base];
            for (long a = 1; a < axis; ++a) mx = fmaxf(mx, x[base + a * inner]);
            float sum = 0;
            for (long a = 0; a < axis; ++a) {
                const float v = expf(x[base + a * inner] - mx);
                y[base + a * inner] = v;
                sum += v;
            }
            for (long a = 0; a < axis; ++a) y[base + a * inner] /= sum;
        }
}

/* QuantizeLinear fp32 -> 8-bit (templates/quantize_linear_op.c.j2): scale and
 * zero point per tensor (axis_len 1) or per index along an axis. */
void orc_quantize_linear(const float *x, const float *scale, const uint8_t *zp, int zp_signed, int y_signed,
                         long outer, long axis_len, long inner, uint8_t *y)
{
    const float lo = y_signed ? (float)INT8_MIN : 0.0f, hi = y_signed ? (float)INT8_MAX : (float)UINT8_MAX;
    for (long o = 0; o < outer; ++o)
        for (long a = 0; a < axis_len; ++a)
            for (long i = 0; i < inner; ++i) {
                const long idx = (o * axis_len + a) * inner + i;
                const float z = zp ? (zp_signed ? (float)(int8_t)zp[a] : (float)zp[a]) : 0.0f;
                const float scaled = x[idx] / scale[a];
                float r = nearbyintf(scaled) + z;
                r = fmaxf(r, lo);
                r = fminf(r, hi);
                y[idx] = y_signed ? (uint8_t)(int8_t)r : (uint8_t)r;
            }
}

/* DequantizeLinear 8-bit -> fp32 (templates/dequantize_linear_op.c.j2). */
void orc_dequantize_linear(const uint8_t *x, int x_signed, const float *scale, const uint8_t *zp,
                           long outer, long axis_len, long inner, float *y)
{
    for (long o = 0; o < outer; ++o)
        for (long a = 0; a < axis_len; ++a)
            for (long i = 0; i < inner; ++i) {
                const long idx = (o * axis_len + a) * inner + i;
                const float xv = x_signed ? (float)(int8_t)x[idx] : (float)x[idx];
                const float z = zp ? (x_signed ? (float)(int8_t)zp[a] : (float)zp[a]) : 0.0f;
                y[idx] = (xv - z) * scale[a];
            }
}

/* ---------------------------------------------------------------------------
 * MaxPool, 2-D NCHW, 8-bit, no indices (templates/maxpool_op.c.j2:30-66):
 * start from the type's minimum, max over the in-bounds taps.
 * ------------------------------------------------------------------------- */
void orc_maxpool8(const uint8_t *x, uint8_t *y, int is_signed, long n, long c, long h, long w, long oh, long ow,
                  long kh, long kw, long sh, long sw, long dh, long dw, long pt, long pl)
{
    for (long b = 0; b < n * c; ++b)
        for (long oy = 0; oy < oh; ++oy)
            for (long ox = 0; ox < ow; ++ox) {
                int m = is_signed ? INT8_MIN : 0;
                for (long ky = 0; ky < kh; ++ky) {
                    const long iy = oy * sh + ky * dh - pt;
                    if (iy < 0 || iy >= h) continue;
                    for (long kx = 0; kx < kw; ++kx) {
                        const long ix = ox * sw + kx * dw - pl;
                        if (ix < 0 || ix >= w) continue;
                        const uint8_t raw = x[(b * h + iy) * w + ix];
                        const int v = is_signed ? (int)(int8_t)raw : (int)raw;
                        m = v > m ? v : m;
                    }
                }
                y[(b * oh + oy) * ow + ox] = (uint8_t)m;
            }
}

/* ---------------------------------------------------------------------------
 * QLinearAveragePool, 2-D NCHW, float compute (templates/qlinear_average_pool_op.c.j2:1-3,
 * :165-189): int32 sum of (x - zx) over the in-bounds taps, denominator the tap
 * count (or KH*KW with count_include_pad), mean = (float)acc / (float)denom,
 * y = clamp((int32_t)roundf(mean * scale) + zy), scale = (float)xs / (float)ys.
 * ------------------------------------------------------------------------- */
void orc_qavgpool8(const uint8_t *x, uint8_t *y, int x_signed, int y_signed, long n, long c, long h, long w,
                   long oh, long ow, long kh, long kw, long sh, long sw, long dh, long dw, long pt, long pl,
                   int count_include_pad, float x_scale, int x_zero, float y_scale, int y_zero)
{
    const float scale = ((float)x_scale) / ((float)y_scale);
    const int lo = y_signed ? INT8_MIN : 0, hi = y_signed ? INT8_MAX : UINT8_MAX;
    for (long b = 0; b < n * c; ++b)
        for (long oy = 0; oy < oh; ++oy)
            for (long ox = 0; ox < ow; ++ox) {
                int32_t acc = 0;
                long count = 0;
                for (long ky = 0; ky < kh; ++ky) {
                    const long iy = oy * sh + ky * dh - pt;
                    for (long kx = 0; kx < kw; ++kx) {
                        const long ix = ox * sw + kx * dw - pl;
                        if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
                            const uint8_t raw = x[(b * h + iy) * w + ix];
                            acc += (x_signed ? (int32_t)(int8_t)raw : (int32_t)raw) - x_zero;
                            ++count;
                        } else if (count_include_pad) {
                            ++count;
                        }
                    }
                }
                const long denom = count_include_pad ? kh * kw : count;
                float mean = (denom > 0) ? (((float)acc) / (float)denom) : (float)0;
                int32_t r = (int32_t)roundf(mean * scale) + y_zero;
                r = r < lo ? lo : r;
                r = r > hi ? hi : r;
                y[(b * oh + oy) * ow + ox] = (uint8_t)r;
            }
}

/* ---------------------------------------------------------------------------
 * QLinearSoftmax, 8-bit (templates/qlinear_softmax_op.c.j2:1-54): v = (float)(x - zx)
 * * xs, max with fmaxf, sum of expf(v - max) in axis order, y = clamp(nearbyintf(
 * (expf(v - max) * inv) / sum) + zy) with inv = floorf(1 / ys).
 * ------------------------------------------------------------------------- */
void orc_qsoftmax8(const uint8_t *x, uint8_t *y, int x_signed, int y_signed, long outer, long axis, long inner,
                   float x_scale, int x_zero, float y_scale, int y_zero)
{
    const float zy = (float)y_zero;
    const float lo = y_signed ? (float)INT8_MIN : 0.0f, hi = y_signed ? (float)INT8_MAX : (float)UINT8_MAX;
    const float inv = floorf((float)1 / y_scale);
#define ORC_QS_V(i) (((float)((x_signed ? (int32_t)(int8_t)x[i] : (int32_t)x[i]) - x_zero)) * x_scale)
    for (long o = 0; o < outer; ++o)
        for (long in = 0; in < inner; ++in) {
            const long base = o * axis * inner + in;
            float mx = ORC_QS_V(base);
            for (long a = 1; a < axis; ++a) mx = fmaxf(mx, ORC_QS_V(base + a * inner));
            float sum = (float)0;
            for (long a = 0; a < axis; ++a) sum += expf(ORC_QS_V(base + a * inner) - mx);
            for (long a = 0; a < axis; ++a) {
                const float e = expf(ORC_QS_V(base + a * inner) - mx);
                const float scaled = (e * inv) / sum;
                float r = nearbyintf(scaled) + zy;
                r = fmaxf(r, lo);
                r = fminf(r, hi);
                y[base + a * inner] = y_signed ? (uint8_t)(int8_t)r : (uint8_t)r;
            }
        }
#undef ORC_QS_V
}
