/*
 * TEST INFRASTRUCTURE ONLY: C + OpenMP restatement of the reference's quantized decode path, used as the timed CPU
 * baseline and for full-size checks. Not linked into, loaded by or called from the product library.
 *
 * Restates (paths inside the komp project):
 *   orc_quant_q8_0   ktl.q8_0_quantize   patches/0001-language-extra-kurn.patch:104-114, kernels.py:22-33
 *   orc_quant_q8_K   ktl.q8_K_quantize   patch:117-131, kernels.py:36-45, bsums as host.q8_K_blocks host.py:43-52
 *   orc_gemv         exact int block dots (verify.exact_idots, verify.py:94-100) and KURN's reference dot rebuilt
 *                    in f64 in block order (verify.rebuild_reference, verify.py:103-120)
 *
 * Build (oracle/build.py): gcc -O2 -fopenmp -ffp-contract=off -shared -fPIC. No fast-math, no FMA contraction:
 * every float operation is the correctly rounded IEEE operation the reference specifies.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static float bits_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* IEEE binary16 -> binary32, exact. */
float orc_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const int exp = (h >> 10) & 0x1f;
  const uint32_t mant = h & 0x3ff;
  float v;
  if (exp == 0) {
    v = ldexpf((float)mant, -24); /* zero or subnormal */
  } else if (exp == 31) {
    return bits_f32(sign | 0x7f800000u | (mant << 13));
  } else {
    v = ldexpf((float)(mant | 0x400), exp - 25);
  }
  return bits_f32(f32_bits(v) | sign);
}

/* IEEE binary32 -> binary16 with round-to-nearest-even (overflow to inf, gradual underflow). */
uint16_t orc_float_to_half(float f) {
  uint32_t x = f32_bits(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  x &= 0x7fffffffu;
  if (x >= 0x7f800000u) return sign | 0x7c00u | (x > 0x7f800000u ? 0x200u : 0u);
  if (x >= 0x477ff000u) return sign | 0x7c00u; /* >= 65520 rounds to infinity */
  if (x < 0x38800000u) {                      /* below 2^-14: f16 subnormal or zero */
    const float t = nearbyintf(bits_f32(x) * 0x1p24f);
    return sign | (uint16_t)t;                /* 1024 becomes the smallest normal, 0x0400 */
  }
  const uint32_t mant = x & 0x7fffffu;
  const int exp = (int)(x >> 23) - 127 + 15;
  uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
  return sign | (uint16_t)h;
}

void orc_quant_q8_0(const float* x, int64_t M, int64_t K, int8_t* xq, float* xd) {
  const int64_t nb = K / 32;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < M * nb; ++g) {
    const float* v = x + g * 32; /* row-major [M][K]: block g of the flattened array */
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int i = 0; i < 32; ++i) {
      const float p = v[i] * id;
      xq[g * 32 + i] = (int8_t)(int)roundf(p);
    }
    xd[g] = orc_half_to_float(orc_float_to_half(d));
  }
}

void orc_quant_q8_K(const float* x, int64_t M, int64_t K, int8_t* xq, float* xd, int16_t* bsums) {
  const int64_t nb = K / 256;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < M * nb; ++g) {
    const float* v = x + g * 256;
    float amax = 0.0f;
    int first = 0;
    for (int i = 0; i < 256; ++i) {
      const float a = fabsf(v[i]);
      if (a > amax) { /* strict: lowest index among equal magnitudes */
        amax = a;
        first = i;
      }
    }
    const int nz = amax != 0.0f;
    const float iscale = -127.0f / (nz ? v[first] : 1.0f);
    for (int i = 0; i < 256; ++i) {
      float q = nearbyintf(iscale * v[i]);
      if (q > 127.0f) q = 127.0f;
      xq[g * 256 + i] = nz ? (int8_t)(int)q : 0;
    }
    xd[g] = nz ? 1.0f / iscale : 0.0f;
    if (bsums) {
      for (int j = 0; j < 16; ++j) {
        int s = 0;
        for (int i = 0; i < 16; ++i) s += xq[g * 256 + j * 16 + i];
        bsums[g * 16 + j] = (int16_t)s;
      }
    }
  }
}

/* Exact int32 dot of one Q4_0 block (16 quant bytes) with 32 int8 activations. */
static int32_t dot_q4_0(const uint8_t* q, const int8_t* x) {
  int32_t s = 0;
  for (int i = 0; i < 16; ++i) s += ((int32_t)(q[i] & 15) - 8) * x[i] + ((int32_t)(q[i] >> 4) - 8) * x[i + 16];
  return s;
}

/* Exact int32 dot of one TQ2_0 block (64 quant bytes) with 256 int8 activations: byte h*32+i, bits 2j hold value
 * h*128 + j*32 + i. */
static int32_t dot_tq2_0(const uint8_t* q, const int8_t* x) {
  int32_t s = 0;
  for (int h = 0; h < 2; ++h)
    for (int j = 0; j < 4; ++j)
      for (int i = 0; i < 32; ++i) s += ((int32_t)((q[h * 32 + i] >> (2 * j)) & 3) - 1) * x[h * 128 + j * 32 + i];
  return s;
}

/* Exact int32 dot of one Q8_0 block (32 int8 weights) with 32 int8 activations (an extension: ggml block_q8_0). */
static int32_t dot_q8_0(const uint8_t* q, const int8_t* x) {
  int32_t s = 0;
  for (int i = 0; i < 32; ++i) s += (int32_t)(int8_t)q[i] * x[i];
  return s;
}

/* ggml's IQ4_NL levels (kvalues_iq4nl): nibble -> int8 value. */
static const int8_t kIq4nlLevels[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* Exact int32 dot of one IQ4_NL block (16 nibble bytes laid out as Q4_0's) with 32 int8 activations (an extension:
 * ggml block_iq4_nl, level[nibble] in place of nibble - 8). */
static int32_t dot_iq4_nl(const uint8_t* q, const int8_t* x) {
  int32_t s = 0;
  for (int i = 0; i < 16; ++i) s += (int32_t)kIq4nlLevels[q[i] & 15] * x[i] + (int32_t)kIq4nlLevels[q[i] >> 4] * x[i + 16];
  return s;
}

/*
 * One Q4_K super-block in the split planes (an extension, pinned to gguf-py's Q4_K codec): 128 quant bytes, one
 * 16-byte chunk per 32-value sub-block j laid out as a Q4_0 block (nibbles 0..15, no offset), and the 20-byte scale
 * record (f16 d, f16 dmin, then the bytes sc_j, m_j). *S = sum_j sc_j * dot_j (exact), *MN = sum_j m_j * sum(x_j).
 */
static void dot_q4_k(const uint8_t* q, const uint8_t* rec, const int8_t* x, int32_t* S, int32_t* MN) {
  int32_t st = 0, mt = 0;
  for (int j = 0; j < 8; ++j) {
    int32_t d = 0, sx = 0;
    for (int i = 0; i < 16; ++i) {
      d += (int32_t)(q[16 * j + i] & 15) * x[32 * j + i] + (int32_t)(q[16 * j + i] >> 4) * x[32 * j + i + 16];
      sx += x[32 * j + i] + x[32 * j + i + 16];
    }
    st += (int32_t)rec[4 + 2 * j] * d;
    mt += (int32_t)rec[5 + 2 * j] * sx;
  }
  *S = st;
  *MN = mt;
}

/*
 * y[m][n] = KURN reference dot (f64, sequential over blocks; q4_0 / q8_0 / iq4_nl: (dw*dx)*s, tq2_0: (dx*dw)*s, dx of
 * q8_0 activations read back as its f16), s (nullable) = int32 block dots [M][N][nb]. fmt: 0 Q4_0, 1 TQ2_0, 2 Q8_0,
 * 3 IQ4_NL, 4 Q4_K (ws: 20-byte records, row stride nb * 10; y = sum over super-blocks of dx * (d * S - dmin * MN)
 * in f64, s = S).
 * nthreads <= 0 uses the OpenMP default.
 */
static void orc_gemv_q4_k(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd,
                          int64_t N, int64_t K, int64_t M, double* y, int32_t* s) {
  const int64_t nb = K / 256;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const uint8_t* row = wq + n * ldwq;
    const uint8_t* recs = (const uint8_t*)(ws + n * nb * 10);
    for (int64_t m = 0; m < M; ++m) {
      double total = 0.0;
      for (int64_t b = 0; b < nb; ++b) {
        int32_t S, MN;
        const uint8_t* rec = recs + b * 20;
        dot_q4_k(row + b * 128, rec, xq + m * K + b * 256, &S, &MN);
        if (s) s[(m * N + n) * nb + b] = S;
        uint16_t dh, mh;
        memcpy(&dh, rec, 2);
        memcpy(&mh, rec + 2, 2);
        const double d = (double)orc_half_to_float(dh), dmin = (double)orc_half_to_float(mh);
        total += (double)xd[m * nb + b] * (d * (double)S - dmin * (double)MN);
      }
      y[m * N + n] = total;
    }
  }
}

void orc_gemv(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd,
              int64_t N, int64_t K, int64_t M, double* y, int32_t* s, int nthreads) {
  const int blk = fmt == 1 ? 256 : 32;
  const int qb = (fmt == 0 || fmt == 3) ? 16 : fmt == 1 ? 64 : 32;
  const int64_t nb = K / blk;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  if (fmt == 4) {
    orc_gemv_q4_k(wq, ldwq, ws, xq, xd, N, K, M, y, s);
    return;
  }
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const uint8_t* row = wq + n * ldwq;
    for (int64_t m = 0; m < M; ++m) {
      const int8_t* xr = xq + m * K;
      double total = 0.0;
      for (int64_t b = 0; b < nb; ++b) {
        const int32_t d = fmt == 0   ? dot_q4_0(row + b * qb, xr + b * blk)
                          : fmt == 1 ? dot_tq2_0(row + b * qb, xr + b * blk)
                          : fmt == 3 ? dot_iq4_nl(row + b * qb, xr + b * blk)
                                     : dot_q8_0(row + b * qb, xr + b * blk);
        if (s) s[(m * N + n) * nb + b] = d;
        const double dw = (double)orc_half_to_float((uint16_t)ws[n * nb + b]);
        double dx = (double)xd[m * nb + b];
        if (fmt != 1) dx = (double)orc_half_to_float(orc_float_to_half(xd[m * nb + b]));
        const double scale = fmt != 1 ? dw * dx : dx * dw;
        total += scale * (double)d;
      }
      y[m * N + n] = total;
    }
  }
}

/* Sets the OpenMP team size of every later call (the quantizers' and the GEMV's parallel loops). Callers pass the
 * number of cores this process may run on, so an inherited OMP_NUM_THREADS=1 (torchrun sets it) does not serialize
 * the baseline. */
void orc_set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
