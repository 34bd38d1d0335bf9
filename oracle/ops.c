/* CPU oracle: plain-C restatement of the reference engine's kernels.
 *
 * TEST INFRASTRUCTURE ONLY. Used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py as the checker; the product never links it.
 *
 * Each function restates one Triton kernel of the reference
 * (python/cutriton/triton_kernels/resnet.py, transformer.py) with the same
 * arithmetic: same accumulation order (serial over k), FP32 accumulators,
 * FP16 inputs widened to FP32, round-to-nearest-even FP16 stores. Sizes are
 * meant for seconds of CPU time. Compiled by oracle/Makefile into
 * oracle/_build/liboracle.so and called through ctypes.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ---- IEEE binary16 <-> binary32 ------------------------------------------ */

float oracle_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else { /* subnormal: normalise */
    int shift = 0;
    while ((man & 0x400u) == 0) {
      man <<= 1;
      ++shift;
    }
    bits = sign | ((uint32_t)(113 - shift) << 23) | ((man & 0x3FFu) << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

/* Round-to-nearest-even binary64 -> binary16 (overflow to inf, NaN kept).
 * Any float, and the exact sum of two halves, is exact in binary64, so this
 * single rounding is the correctly rounded FP16 result. */
static uint16_t double_to_half(double d) {
  uint16_t sign = signbit(d) ? 0x8000u : 0u;
  double a = fabs(d);
  if (isnan(d)) return (uint16_t)(sign | 0x7E00u);
  if (isinf(a)) return (uint16_t)(sign | 0x7C00u);
  if (a == 0.0) return sign;
  int e2;
  frexp(a, &e2);                 /* a = f * 2^e2, f in [0.5, 1) */
  int exponent = e2 - 1;         /* floor(log2 a) */
  if (exponent < -14) exponent = -14;
  double quantum = ldexp(1.0, exponent - 10);
  double steps = nearbyint(a / quantum); /* exact division; ties to even */
  if (steps >= 2048.0) {
    steps /= 2.0;
    exponent += 1;
  }
  if (exponent > 15) return (uint16_t)(sign | 0x7C00u);
  uint32_t n = (uint32_t)steps;
  if (n < 1024u) return (uint16_t)(sign | n); /* subnormal (exponent == -14) */
  return (uint16_t)(sign | ((uint32_t)(exponent + 15) << 10) | (n - 1024u));
}

uint16_t oracle_float_to_half(float f) { return double_to_half((double)f); }

static float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f)); }

/* ---- ResNet family (resnet.py) --------------------------------------------- */

/* Direct convolution over NCHW/OIHW with the reference's loop order
 * (resnet.py:28-40): for each output, one serial sum over (c, r, s).
 * mode 0: raw conv; 1: + BN; 2: + BN + ReLU; 3: + BN + residual + ReLU
 * (BN as (acc - mean) * rsqrt(var + eps) * scale + bias, resnet.py:41-47). */
void oracle_conv2d(const float* x, const float* w, const float* scale, const float* bias,
                   const float* mean, const float* var, const float* residual, float* y, int n, int c,
                   int h, int wd, int k, int r, int s, int oh, int ow, int sh, int sw, int ph, int pw,
                   int dh, int dw, float eps, int mode) {
  for (int b = 0; b < n; ++b)
    for (int oc = 0; oc < k; ++oc)
      for (int i = 0; i < oh; ++i)
        for (int j = 0; j < ow; ++j) {
          float acc = 0.0f;
          for (int ic = 0; ic < c; ++ic)
            for (int kh = 0; kh < r; ++kh)
              for (int kw = 0; kw < s; ++kw) {
                int ih = i * sh - ph + kh * dh;
                int iw = j * sw - pw + kw * dw;
                float xv = 0.0f;
                if (ih >= 0 && ih < h && iw >= 0 && iw < wd) xv = x[(((long)b * c + ic) * h + ih) * wd + iw];
                acc = fmaf(xv, w[(((long)oc * c + ic) * r + kh) * s + kw], acc);
              }
          long at = (((long)b * k + oc) * oh + i) * ow + j;
          float v = acc;
          if (mode >= 1) v = (v - mean[oc]) * (1.0f / sqrtf(var[oc] + eps)) * scale[oc] + bias[oc];
          if (mode == 3) v += residual[at];
          if (mode >= 2) v = v > 0.0f ? v : 0.0f;
          y[at] = v;
        }
}

void oracle_batch_norm(const float* x, const float* scale, const float* bias, const float* mean,
                       const float* var, float* y, long total, int channels, int spatial, float eps) {
  for (long i = 0; i < total; ++i) {
    int ch = (int)((i / spatial) % channels);
    y[i] = (x[i] - mean[ch]) * (1.0f / sqrtf(var[ch] + eps)) * scale[ch] + bias[ch];
  }
}

void oracle_relu(const float* x, float* y, long total) {
  for (long i = 0; i < total; ++i) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

void oracle_add(const float* a, const float* b, float* y, long total) {
  for (long i = 0; i < total; ++i) y[i] = a[i] + b[i];
}

void oracle_add_relu(const float* a, const float* b, float* y, long total) {
  for (long i = 0; i < total; ++i) {
    float v = a[i] + b[i];
    y[i] = v > 0.0f ? v : 0.0f;
  }
}

/* resnet.py:159-182: out-of-range taps are -inf; pads[0]/pads[1] are top/left. */
void oracle_max_pool(const float* x, float* y, int n, int c, int h, int w, int oh, int ow, int kh_, int kw_,
                     int sh, int sw, int ph, int pw, int dh, int dw) {
  for (long p = 0; p < (long)n * c; ++p)
    for (int i = 0; i < oh; ++i)
      for (int j = 0; j < ow; ++j) {
        float best = -INFINITY;
        for (int a = 0; a < kh_; ++a)
          for (int b = 0; b < kw_; ++b) {
            int ih = i * sh - ph + a * dh;
            int iw = j * sw - pw + b * dw;
            if (ih < 0 || ih >= h || iw < 0 || iw >= w) continue;
            float v = x[(p * h + ih) * w + iw];
            if (v > best) best = v;
          }
        y[(p * oh + i) * ow + j] = best;
      }
}

/* resnet.py:185-198: serial sum over H*W, then divide. */
void oracle_global_average_pool(const float* x, float* y, int n, int c, int h, int w) {
  int spatial = h * w;
  for (long p = 0; p < (long)n * c; ++p) {
    float acc = 0.0f;
    for (int i = 0; i < spatial; ++i) acc += x[p * spatial + i];
    y[p] = acc / (float)spatial;
  }
}

/* resnet.py:201-213: C = A . B, serial k sum, FP32. */
void oracle_gemm_f32(const float* a, const float* b, float* y, int m, int n, int k) {
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) {
      float acc = 0.0f;
      for (int t = 0; t < k; ++t) acc = fmaf(a[(long)i * k + t], b[(long)t * n + j], acc);
      y[(long)i * n + j] = acc;
    }
}

/* ---- Transformer family (transformer.py) ---------------------------------- */

/* transformer.py:17-107: FP32 accumulation over k of FP16 products; GELU (if
 * gelu != 0) on the FP32 accumulator; round-to-nearest FP16 store. */
void oracle_gemm_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, int m, int n, int k, int gelu) {
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) {
      float acc = 0.0f;
      for (int t = 0; t < k; ++t)
        acc = fmaf(oracle_half_to_float(a[(long)i * k + t]), oracle_half_to_float(b[(long)t * n + j]), acc);
      y[(long)i * n + j] = oracle_float_to_half(gelu ? gelu_erf(acc) : acc);
    }
}

void oracle_gelu_f16(const uint16_t* x, uint16_t* y, long total) {
  for (long i = 0; i < total; ++i) y[i] = oracle_float_to_half(gelu_erf(oracle_half_to_float(x[i])));
}

/* FP16 addition (transformer.py:119-125): the exact sum rounded once to
 * FP16, which is what FP16 hardware addition returns. */
void oracle_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, long total) {
  for (long i = 0; i < total; ++i) {
    y[i] = double_to_half((double)oracle_half_to_float(a[i]) + (double)oracle_half_to_float(b[i]));
  }
}

static void norm_row(float* v, int columns, float eps, const uint16_t* scale, const uint16_t* bias, uint16_t* out) {
  float sum = 0.0f;
  for (int j = 0; j < columns; ++j) sum += v[j];
  float mean = sum / (float)columns;
  float sq = 0.0f;
  for (int j = 0; j < columns; ++j) {
    v[j] -= mean;
    sq += v[j] * v[j];
  }
  float var = sq / (float)columns;
  float inv = 1.0f / sqrtf(var + eps);
  for (int j = 0; j < columns; ++j)
    out[j] = oracle_float_to_half(v[j] * inv * oracle_half_to_float(scale[j]) + oracle_half_to_float(bias[j]));
}

/* transformer.py:128-149 (residual == NULL) and 152-177 (FP32 x + residual). */
void oracle_layer_norm_f16(const uint16_t* x, const uint16_t* residual, const uint16_t* scale,
                           const uint16_t* bias, uint16_t* y, int rows, int columns, float eps, float* scratch) {
  for (int r = 0; r < rows; ++r) {
    for (int j = 0; j < columns; ++j) {
      float v = oracle_half_to_float(x[(long)r * columns + j]);
      if (residual) v += oracle_half_to_float(residual[(long)r * columns + j]);
      scratch[j] = v;
    }
    norm_row(scratch, columns, eps, scale, bias, y + (long)r * columns);
  }
}

/* transformer.py:180-190. */
void oracle_softmax_f16(const uint16_t* x, uint16_t* y, int rows, int columns) {
  for (int r = 0; r < rows; ++r) {
    float peak = -INFINITY;
    for (int j = 0; j < columns; ++j) {
      float v = oracle_half_to_float(x[(long)r * columns + j]);
      if (v > peak) peak = v;
    }
    float sum = 0.0f;
    for (int j = 0; j < columns; ++j) sum += expf(oracle_half_to_float(x[(long)r * columns + j]) - peak);
    for (int j = 0; j < columns; ++j)
      y[(long)r * columns + j] = oracle_float_to_half(expf(oracle_half_to_float(x[(long)r * columns + j]) - peak) / sum);
  }
}
