/*
 * CPU oracle for the Q4 KV-cache attention path.  TEST INFRASTRUCTURE ONLY:
 * tests, the smoke check and bench.py's CPU-baseline leg may call this code;
 * the product path (agent-memory_b200) never does.
 *
 * What it restates, and from where:
 *
 *  - Affine 4-bit quantization with group size 64 (mx.quantize, mlx 0.30.3,
 *    the CPU backend's affine quantizer).  The reference calls it at
 *    src/agent_memory/adapters/outbound/mlx_quantized_extensions.py:273-274
 *    (quantize-on-append), application/batch_engine.py:1948-1949 (block
 *    extraction) and safetensors_cache_adapter.py:177-178.  mlx is a
 *    third-party dependency (pyproject.toml:33) that is not vendored in the
 *    reference; its published algorithm, restated here, is per 64-element
 *    group in fp32:
 *        scale = max((max - min) / 15, 1e-7)
 *        if |min| > |max|: edge = min            else: edge = max, scale = -scale
 *        q0 = rint(edge / scale)
 *        if q0 != 0: scale = edge / q0, bias = edge    else: bias = 0
 *        code = clamp(rint((w - bias) / scale), 0, 15)
 *    scale and bias are then rounded to the input dtype (fp16 or bf16,
 *    tests/mlx/test_real_cache_round_trip.py:329-337 pins that rule).
 *    In the mlx sources the rule lives in mlx/backend/cpu/quantized.cpp
 *    (CPU backend) and in the Metal kernels' affine_quantize
 *    (mlx/backend/metal/kernels/quantized.h).  Details this restatement
 *    fixes and the tests pin against the GPU kernel bit-for-bit: ties of
 *    (w - bias) / scale round to the even code (rint), divisions are IEEE
 *    round-to-nearest, codes come from the fp32 scale and bias before they
 *    are rounded to the storage dtype, all-zero groups keep bias 0 and the
 *    scale floor (stored in fp16 as the subnormal 1.19e-7), subnormal inputs
 *    are not flushed.  Groups whose fp32 range or edge / 1e-7 overflows
 *    (bf16 values beyond ~1.7e38, or bf16 constants beyond ~3.4e31) have no
 *    defined codes, in mlx as here.
 *    Codes are packed 8 per uint32, element d in word d/8 at bits 4*(d%8)
 *    (mlx_fused_attention.py:274-288 reads them that way).
 *
 *  - Dequantization x = code * scale + bias in fp32
 *    (mlx_fused_attention.py:274-288, the reference's dequant4()).
 *
 *  - Scaled dot-product attention over a Q4 cache with the reference's op
 *    order (mlx_fused_attention.py:69-139): scores = (scale*q) . k^T, a
 *    boolean mask replaces masked scores by the dtype minimum while an
 *    additive mask is added, softmax in fp32, then P . V.  GQA maps query
 *    head h to KV head h / n_rep (mlx_fused_attention.py:79, :304).  The
 *    structured mask (causal offset, sliding window, left padding) is
 *    mlx-lm's create_causal_mask as called at
 *    mlx_quantized_extensions.py:483 and :601-615: query l of L sits at
 *    position kv_len - L + l and sees key r when
 *        kv_start <= r <= pos  and (window == 0 or r > pos - window).
 *    Masked-but-present keys take the finite minimum score, as the
 *    reference's where(mask, s, finfo.min) does, so a fully masked row
 *    averages V uniformly exactly like the reference.
 *
 * Parity status: the quantizer restates mlx's published algorithm; no
 * golden vector produced by mlx itself exists in this environment (mlx is
 * not installed), so bit-exactness against mlx is UNPINNED.  The reference
 * tests pin only dtypes, shapes, the Q4 byte formula and persistence
 * bit-identity, and the oracle is checked against those.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef __AVX2__
#include <immintrin.h>
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

enum { AMO_F16 = 0, AMO_BF16 = 1, AMO_F32 = 2 };
enum { AMO_CONTIGUOUS = 0, AMO_PAGED = 1 };
enum { AMO_MASK_NONE = 0, AMO_MASK_BOOL = 1, AMO_MASK_ADDITIVE = 2 };

/* ---- 16-bit float conversions (IEEE binary16 / bfloat16, round to nearest even) ---- */

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do { man <<= 1; e++; } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) { /* inf / nan */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  }
  if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
    return (uint16_t)(sign | 0x7c00u);
  }
  if (ax < 0x33000001u) { /* < 2^-25 (+tiny): rounds to zero */
    return (uint16_t)sign;
  }
  int e = (int)(ax >> 23) - 127;
  uint32_t man = (ax & 0x7fffffu) | 0x800000u;
  uint32_t h;
  if (e < -14) { /* subnormal half */
    int shift = -14 - e + 13;
    uint32_t q = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    h = q;
  } else {
    uint32_t q = man >> 13;
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    h = ((uint32_t)(e + 15) << 10) + (q - 0x400u);
    if (q == 0x800u) h = ((uint32_t)(e + 16) << 10); /* mantissa overflow */
  }
  return (uint16_t)(sign | h);
}

static float bf16_to_f32(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}

static inline float h2f(uint16_t v, int dtype) {
  return dtype == AMO_BF16 ? bf16_to_f32(v) : f16_to_f32(v);
}

static inline uint16_t f2h(float v, int dtype) {
  return dtype == AMO_BF16 ? f32_to_bf16(v) : f32_to_f16(v);
}

int amo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void amo_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

void amo_f16_to_f32(const uint16_t* in, int dtype, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = h2f(in[i], dtype);
}

void amo_f32_to_f16(const float* in, int dtype, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; i++) out[i] = f2h(in[i], dtype);
}

/* ---- quantization of one 64-element group (mlx affine, bits=4) ---- */

static void quantize_group(const float* w, uint32_t* codes /* 8 words */, float* out_scale,
                           float* out_bias) {
  const float n_bins = 15.0f;
  const float eps = 1e-7f;
  float w_min = INFINITY, w_max = -INFINITY;
  for (int j = 0; j < 64; j++) {
    w_max = fmaxf(w_max, w[j]);
    w_min = fminf(w_min, w[j]);
  }
  int side = fabsf(w_min) > fabsf(w_max);
  float scale = fmaxf((w_max - w_min) / n_bins, eps);
  scale = side ? scale : -scale;
  float edge = side ? w_min : w_max;
  float q0 = rintf(edge / scale);
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = edge / q0;
    bias = edge;
  }
  for (int word = 0; word < 8; word++) {
    uint32_t packed = 0;
    for (int k = 0; k < 8; k++) {
      float v = rintf((w[word * 8 + k] - bias) / scale);
      v = fminf(fmaxf(v, 0.0f), n_bins);
      packed |= (uint32_t)v << (4 * k);
    }
    codes[word] = packed;
  }
  *out_scale = scale;
  *out_bias = bias;
}

/* x: [rows, dim] 16-bit floats of `dtype`; codes [rows, dim/8]; scales/biases [rows, dim/64]. */
void amo_quantize(const uint16_t* x, int dtype, int64_t rows, int dim, uint32_t* codes,
                  uint16_t* scales, uint16_t* biases) {
  const int ng = dim / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    float w[64];
    for (int g = 0; g < ng; g++) {
      for (int j = 0; j < 64; j++) w[j] = h2f(x[r * dim + g * 64 + j], dtype);
      float s, b;
      quantize_group(w, codes + r * (dim / 8) + g * 8, &s, &b);
      scales[r * ng + g] = f2h(s, dtype);
      biases[r * ng + g] = f2h(b, dtype);
    }
  }
}

/* Same rule over fp32 input (used by the oracle to quantize data held as float). */
void amo_quantize_f32(const float* x, int out_dtype, int64_t rows, int dim, uint32_t* codes,
                      uint16_t* scales, uint16_t* biases) {
  const int ng = dim / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    for (int g = 0; g < ng; g++) {
      float s, b;
      quantize_group(x + r * dim + g * 64, codes + r * (dim / 8) + g * 8, &s, &b);
      scales[r * ng + g] = f2h(s, out_dtype);
      biases[r * ng + g] = f2h(b, out_dtype);
    }
  }
}

static inline void dequant_row(const uint32_t* codes, const uint16_t* scales,
                               const uint16_t* biases, int sdtype, int dim, float* out) {
  for (int g = 0; g < dim / 64; g++) {
    float s = h2f(scales[g], sdtype);
    float b = h2f(biases[g], sdtype);
#ifdef __AVX2__
    /* the 8 codes of a word: one broadcast, one variable shift per lane, a mask, a convert
       and one fused multiply-add (code * scale + bias, fp32) */
    const __m256i shifts = _mm256_setr_epi32(0, 4, 8, 12, 16, 20, 24, 28);
    const __m256i nib = _mm256_set1_epi32(15);
    const __m256 vs = _mm256_set1_ps(s), vb = _mm256_set1_ps(b);
    for (int word = 0; word < 8; word++) {
      const __m256i c = _mm256_and_si256(
          _mm256_srlv_epi32(_mm256_set1_epi32((int)codes[g * 8 + word]), shifts), nib);
      _mm256_storeu_ps(out + g * 64 + word * 8, _mm256_fmadd_ps(_mm256_cvtepi32_ps(c), vs, vb));
    }
#else
    for (int word = 0; word < 8; word++) {
      uint32_t w = codes[g * 8 + word];
      for (int k = 0; k < 8; k++) out[g * 64 + word * 8 + k] = (float)((w >> (4 * k)) & 0xfu) * s + b;
    }
#endif
  }
}

void amo_dequantize(const uint32_t* codes, const uint16_t* scales, const uint16_t* biases,
                    int sdtype, int64_t rows, int dim, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++)
    dequant_row(codes + r * (dim / 8), scales + r * (dim / 64), biases + r * (dim / 64), sdtype,
                dim, out + r * dim);
}

/* ---- attention over a Q4 cache ---- */

typedef struct {
  const uint32_t* codes;
  const uint16_t* scales;
  const uint16_t* biases;
  int dim;
} amo_q4_tensor;

/* Row index of (seq b, kv head h, position t) in either layout; -1 when the block id is bad. */
static inline int64_t cache_row(int layout, int64_t cap, int block_tokens, const int32_t* table,
                                int table_stride, int hkv, int b, int h, int64_t t) {
  if (layout == AMO_CONTIGUOUS) return ((int64_t)b * hkv + h) * cap + t;
  int32_t blk = table[(int64_t)b * table_stride + t / block_tokens];
  if (blk < 0 || blk >= cap) return -1;
  return ((int64_t)blk * hkv + h) * block_tokens + t % block_tokens;
}

/*
 * q:    [B, Hq, L, Dk] fp32 (already converted from the query dtype), contiguous.
 * out:  [B, Hq, L, Dv] fp32.
 * mask: optional dense mask as fp32 with element strides (b, h, l, n); stride 0 broadcasts.
 *       AMO_MASK_BOOL treats value != 0 as "keep"; AMO_MASK_ADDITIVE adds the value.
 * Query l sits at position kv_len - L + l.  Keys are streamed in blocks of 256 with a
 * running max per query row (exact softmax up to fp32 rounding).  Accumulation is fp32.
 * Work is split over (sequence, KV head, block of 64 query rows); query rows of one KV
 * head are (l, head-in-group) pairs, so each dequantized key row is shared by all of
 * them, as in the reference's GQA reshape (mlx_fused_attention.py:76-79).
 * Returns 0, or -1 when a block-table entry is out of range (that key is skipped).
 */
int amo_attention(const float* q, int B, int Hq, int L, int Hkv, int Dk, int Dv,
                  const uint32_t* kc, const uint16_t* ks, const uint16_t* kb,
                  const uint32_t* vc, const uint16_t* vs, const uint16_t* vb, int sdtype,
                  int layout, int64_t cap, int block_tokens, const int32_t* table,
                  int table_stride, const int32_t* kv_len, const int32_t* kv_start, int causal,
                  int window, int mask_kind, const float* mask, int64_t msb, int64_t msh,
                  int64_t msl, int64_t msn, float scale, const float* sinks, float* out) {
  const int n_rep = Hq / Hkv;
  const int rows_per_head = n_rep * L;
  const int RB = 64;  /* query rows per work item */
  const int KB = 256; /* keys per streamed block */
  const int n_rb = (rows_per_head + RB - 1) / RB;
  const float masked_score = -65504.0f; /* finfo(float16).min, the reference's masked value */
  int bad = 0;
#pragma omp parallel for collapse(3) schedule(dynamic, 1) reduction(| : bad)
  for (int b = 0; b < B; b++) {
    for (int hk = 0; hk < Hkv; hk++) {
      for (int rb = 0; rb < n_rb; rb++) {
        const int n = kv_len[b];
        const int start = kv_start ? kv_start[b] : 0;
        const int r0 = rb * RB;
        const int nr = rows_per_head - r0 < RB ? rows_per_head - r0 : RB;
        float* kbuf = (float*)malloc(sizeof(float) * (size_t)KB * Dk);
        float* vbuf = (float*)malloc(sizeof(float) * (size_t)KB * Dv);
        char* valid = (char*)malloc((size_t)KB);
        float* sbuf = (float*)malloc(sizeof(float) * KB);
        float* acc = (float*)calloc((size_t)nr * Dv, sizeof(float));
        float* mrow = (float*)malloc(sizeof(float) * nr);
        float* lrow = (float*)calloc((size_t)nr, sizeof(float));
        for (int r = 0; r < nr; r++) mrow[r] = -INFINITY;
        for (int t0 = 0; t0 < n; t0 += KB) {
          const int nt = n - t0 < KB ? n - t0 : KB;
          for (int i = 0; i < nt; i++) {
            int64_t row = cache_row(layout, cap, block_tokens, table, table_stride, Hkv, b, hk,
                                    t0 + i);
            valid[i] = row >= 0;
            if (row < 0) {
              bad = 1;
              continue;
            }
            dequant_row(kc + row * (Dk / 8), ks + row * (Dk / 64), kb + row * (Dk / 64), sdtype,
                        Dk, kbuf + (size_t)i * Dk);
            dequant_row(vc + row * (Dv / 8), vs + row * (Dv / 64), vb + row * (Dv / 64), sdtype,
                        Dv, vbuf + (size_t)i * Dv);
          }
          for (int r = 0; r < nr; r++) {
            const int rr = r0 + r;
            const int l = rr / n_rep;
            const int h = hk * n_rep + rr % n_rep;
            const float* qv = q + (((int64_t)b * Hq + h) * L + l) * Dk;
            const int64_t pos = (int64_t)n - L + l;
            float bm = -INFINITY;
            for (int i = 0; i < nt; i++) {
              const int64_t t = t0 + i;
              float s = masked_score;
              int keep = t >= start;
              if (causal && t > pos) keep = 0;
              if (window > 0 && t <= pos - window) keep = 0;
              if (valid[i]) {
                /* eight partial sums (head dims are multiples of 64), so the compiler can keep
                   them in one vector register; fp32 throughout */
                const float* kr = kbuf + (size_t)i * Dk;
                float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                for (int d = 0; d < Dk; d += 8)
                  for (int j = 0; j < 8; j++) part[j] += qv[d + j] * kr[d + j];
                const float dot = ((part[0] + part[4]) + (part[1] + part[5])) +
                                  ((part[2] + part[6]) + (part[3] + part[7]));
                s = dot * scale;
              }
              if (mask_kind != AMO_MASK_NONE) {
                float mv = mask[b * msb + h * msh + l * msl + t * msn];
                if (mask_kind == AMO_MASK_BOOL) {
                  if (mv == 0.0f) keep = 0;
                } else {
                  s += mv;
                }
              }
              if (!keep || !valid[i]) s = masked_score;
              sbuf[i] = s;
              if (s > bm) bm = s;
            }
            const float m_new = bm > mrow[r] ? bm : mrow[r];
            const float alpha = expf(mrow[r] - m_new);
            float* a = acc + (size_t)r * Dv;
            if (alpha != 1.0f)
              for (int d = 0; d < Dv; d++) a[d] *= alpha;
            float lsum = lrow[r] * alpha;
            for (int i = 0; i < nt; i++) {
              const float p = expf(sbuf[i] - m_new);
              lsum += p;
              if (!valid[i]) continue;
              const float* vr = vbuf + (size_t)i * Dv;
              for (int d = 0; d < Dv; d++) a[d] += p * vr[d];
            }
            lrow[r] = lsum;
            mrow[r] = m_new;
          }
        }
        for (int r = 0; r < nr; r++) {
          const int rr = r0 + r;
          const int l = rr / n_rep;
          const int h = hk * n_rep + rr % n_rep;
          float* o = out + (((int64_t)b * Hq + h) * L + l) * Dv;
          /* attention sink: one extra logit per query head (scaled-score units) that joins
             the softmax normaliser and contributes no value */
          float w = 1.0f, den = lrow[r];
          if (sinks) {
            const float m_all = sinks[h] > mrow[r] ? sinks[h] : mrow[r];
            w = mrow[r] == -INFINITY ? 0.0f : expf(mrow[r] - m_all);
            den = lrow[r] * w + expf(sinks[h] - m_all);
          }
          for (int d = 0; d < Dv; d++)
            o[d] = (n > 0 && den > 0.0f) ? acc[(size_t)r * Dv + d] * w / den : 0.0f;
        }
        free(kbuf);
        free(vbuf);
        free(valid);
        free(sbuf);
        free(acc);
        free(mrow);
        free(lrow);
      }
    }
  }
  return bad ? -1 : 0;
}
