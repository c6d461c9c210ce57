/*
 * CPU oracle for the DFC-AdamW step.  TEST INFRASTRUCTURE ONLY: the parity
 * tests, the smoke check and the CPU-baseline leg of the benchmark call this
 * to check (or time beside) the CUDA path; the product never links it.
 *
 * It restates, element by element and in plain C with explicit rounding, the
 * arithmetic of the reference's eager-PyTorch optimizer step
 * (remote/torch_fiber.py:68-117, YellowJune/T3st):
 *
 *   m1  = m * f32(beta1)                          torch_fiber.py:98  mul_(beta1)
 *   m'  = fma(g, f32(1 - beta1), m1)              torch_fiber.py:98  add_(g, alpha=1-beta1)
 *   v1  = v * f32(beta2)                          torch_fiber.py:99  mul_(beta2)
 *   v'  = fma(f32(1 - beta2) * g, g, v1)          torch_fiber.py:99  addcmul_(g, g, value=1-beta2)
 *   den = sqrt(v') / f32(sqrt(bc2)) + f32(eps)    torch_fiber.py:112
 *   p1  = p * f32(1 - lr * wd)                    torch_fiber.py:114-115
 *   p'  = p1 + (f32(-lr / bc1) * m') / den        torch_fiber.py:116 addcdiv_
 *
 * All scalars are formed in double on the host and rounded once to f32, as
 * PyTorch does when a Python float meets an FP32 tensor.  The sign-fiber mode
 * strips bit 31 of the second-moment word before the update and puts it back
 * afterwards (torch_fiber.py:18-19, 90-107).
 *
 * Reduced-precision parameters (bf16/fp16, remote/torch_fiber.py:45, 114-116):
 * the moments stay FP32; PyTorch's CPU kernels compute mul_ and addcdiv_ in
 * FP32 and round once to the parameter type, with m and den rounded to it
 * first (first.to(parameter.dtype), denominator.to(parameter.dtype)):
 *   p1 = lo(p * decay);  p' = lo(p1 + (f32(-lr/bc1) * lo(m')) / lo(den))
 * lo() rounds to nearest even; a NaN becomes the canonical quiet NaN of the
 * type (bf16 0x7FC0, fp16 0x7E00).
 *
 * Two formats have no counterpart in the reference and are specified here:
 *
 * Packed moment word (bf16 high half + 16-bit error-feedback residual low
 * half).  For an FP32 magnitude a (31 bits):
 *     enc(a) = a + ((a & 0x8000) << 1)        for a <= 0x7F800000
 *     enc(a) = 0x7FC00000                     for NaN (canonical quiet NaN)
 * so the high half is a rounded to the nearest bf16 (ties away from zero) and
 * the low half, read as a signed int16, is the residual in units of the FP32
 * ulp: dec(W) = (hi << 16) + (int16)lo, clamped to [0, 0x7F800000] (NaN words,
 * hi > 0x7F80, decode to themselves).  Every 16-bit residual pattern is a
 * valid residual, and dec(enc(a)) == a for every non-NaN FP32 value.  The
 * first moment keeps its sign in bit 31 (a NaN is stored as +NaN, so CPU and
 * GPU NaN patterns agree); the second moment keeps the reference's payload
 * bit in bit 31 and its magnitude in the rest.
 *
 * Compressed gradient with error feedback.  s = g + e, c = high half of
 * enc(s) (bf16, contiguous for the collective), q = low half (the residual
 * field).  The next call recovers e = dec(c, q) - c exactly; e is 0 when c is
 * not finite.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORC_MODE_PLAIN 0
#define ORC_MODE_SIGNFIBER 1
#define ORC_MODE_PACKED 2

/* element types of parameters and gradients */
#define ORC_F32 0
#define ORC_BF16 1
#define ORC_F16 2

typedef struct orc_hyper {
  float beta1;
  float one_minus_beta1;
  float beta2;
  float one_minus_beta2;
  float sqrt_bc2;
  float eps;
  float decay;
  float neg_step_size;
  float grad_scale;
} orc_hyper;

static inline uint32_t f2u(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float x;
  memcpy(&x, &u, 4);
  return x;
}

/* ---- packed word: magnitude encode/decode (31-bit values) ---- */
uint32_t orc_enc_mag(uint32_t a) {
  if (a > 0x7F800000u) return 0x7FC00000u;
  return a + ((a & 0x8000u) << 1);
}

/* signed value -> packed word; NaN becomes the canonical +NaN word */
static inline uint32_t enc_signed_bits(uint32_t b) {
  uint32_t a = b & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return 0x7FC00000u;
  return (b & 0x80000000u) | orc_enc_mag(a);
}

uint32_t orc_dec_mag(uint32_t w) {
  uint32_t hi = w >> 16;
  if (hi > 0x7F80u) return w;
  int32_t r = (int32_t)(hi << 16) + (int32_t)(int16_t)(w & 0xFFFFu);
  if (r < 0) r = 0;
  if (r > 0x7F800000) r = 0x7F800000;
  return (uint32_t)r;
}

uint32_t orc_pack_signed(float x) { return enc_signed_bits(f2u(x)); }

float orc_unpack_signed(uint32_t w) {
  return u2f((w & 0x80000000u) | orc_dec_mag(w & 0x7FFFFFFFu));
}

static inline float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* round to nearest even, NaN -> 0x7FC0 */
static inline uint16_t f32_to_bf16(float x) {
  uint32_t b = f2u(x);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0u;
  return (uint16_t)((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);
}

static inline float f16_to_f32(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

/* round to nearest even (IEEE conversion), NaN -> 0x7E00 */
static inline uint16_t f32_to_f16(float x) {
  if (isnan(x)) return 0x7E00u;
  _Float16 v = (_Float16)x;
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

static inline float load_elem(int dt, const void* base, int64_t i) {
  if (dt == ORC_BF16) return bf16_to_f32(((const uint16_t*)base)[i]);
  if (dt == ORC_F16) return f16_to_f32(((const uint16_t*)base)[i]);
  return ((const float*)base)[i];
}

static inline void store_elem(int dt, void* base, int64_t i, float x) {
  if (dt == ORC_BF16) ((uint16_t*)base)[i] = f32_to_bf16(x);
  else if (dt == ORC_F16) ((uint16_t*)base)[i] = f32_to_f16(x);
  else ((float*)base)[i] = x;
}

/* value of x rounded to the parameter type */
static inline float round_to(int dt, float x) {
  if (dt == ORC_BF16) return bf16_to_f32(f32_to_bf16(x));
  if (dt == ORC_F16) return f16_to_f32(f32_to_f16(x));
  return x;
}

/* ---- one element of the step ---- */
static inline void step_one(int mode, int pdt, const orc_hyper* h, float* p, float gin,
                            uint32_t* mw, uint32_t* vw) {
  float g = gin * h->grad_scale;
  float m, v;
  uint32_t payload = 0;
  if (mode == ORC_MODE_PACKED) {
    m = orc_unpack_signed(*mw);
    payload = *vw & 0x80000000u;
    v = u2f(orc_dec_mag(*vw & 0x7FFFFFFFu));
  } else if (mode == ORC_MODE_SIGNFIBER) {
    m = u2f(*mw);
    payload = *vw & 0x80000000u;
    v = u2f(*vw & 0x7FFFFFFFu);
  } else {
    m = u2f(*mw);
    v = u2f(*vw);
  }
  float m1 = m * h->beta1;
  float m_new = fmaf(g, h->one_minus_beta1, m1);
  float v1 = v * h->beta2;
  float t = h->one_minus_beta2 * g;
  float v_new = fmaf(t, g, v1);

  uint32_t v_store;
  float v_upd;
  if (mode == ORC_MODE_PLAIN) {
    v_store = f2u(v_new);
    v_upd = v_new;
  } else {
    uint32_t mag = f2u(v_new) & 0x7FFFFFFFu;
    v_upd = u2f(mag);
    v_store = payload | (mode == ORC_MODE_PACKED ? orc_enc_mag(mag) : mag);
  }
  float den = sqrtf(v_upd) / h->sqrt_bc2 + h->eps;
  if (pdt == ORC_F32) {
    float p1 = *p * h->decay;
    float upd = (h->neg_step_size * m_new) / den;
    *p = p1 + upd;
  } else {
    float p1 = round_to(pdt, *p * h->decay);
    float upd = (h->neg_step_size * round_to(pdt, m_new)) / round_to(pdt, den);
    *p = round_to(pdt, p1 + upd);
  }
  *mw = (mode == ORC_MODE_PACKED) ? orc_pack_signed(m_new) : f2u(m_new);
  *vw = v_store;
}

/* p: parameters of type pdt, g: gradients of type gdt (ORC_F32/BF16/F16) */
int orc_step(int mode, const orc_hyper* h, void* p, int pdt, const void* g, int gdt, uint32_t* m,
             uint32_t* v, int64_t n) {
  if (mode < 0 || mode > 2 || pdt < 0 || pdt > 2 || gdt < 0 || gdt > 2) return -1;
  for (int64_t i = 0; i < n; ++i) {
    float pv = load_elem(pdt, p, i);
    step_one(mode, pdt, h, &pv, load_elem(gdt, g, i), m + i, v + i);
    store_elem(pdt, p, i, pv);
  }
  return 0;
}

/* ---- packed-word array conversions ---- */
void orc_pack_first(const float* x, uint32_t* w, int64_t n) {
  for (int64_t i = 0; i < n; ++i) w[i] = orc_pack_signed(x[i]);
}
void orc_unpack_first(const uint32_t* w, float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = orc_unpack_signed(w[i]);
}
/* second moment: bit 31 of the input FP32 word is the payload and is kept */
void orc_pack_second(const uint32_t* physical, uint32_t* w, int64_t n) {
  for (int64_t i = 0; i < n; ++i)
    w[i] = (physical[i] & 0x80000000u) | orc_enc_mag(physical[i] & 0x7FFFFFFFu);
}
void orc_unpack_second(const uint32_t* w, uint32_t* physical, int64_t n) {
  for (int64_t i = 0; i < n; ++i)
    physical[i] = (w[i] & 0x80000000u) | orc_dec_mag(w[i] & 0x7FFFFFFFu);
}

/* ---- compressed gradient with error feedback ---- */
static inline float ef_residual(uint16_t c, uint16_t q) {
  uint32_t hm = c & 0x7FFFu;
  if (hm >= 0x7F80u) return 0.0f;
  uint32_t sign = ((uint32_t)c & 0x8000u) << 16;
  float s = u2f(sign | orc_dec_mag((hm << 16) | q));
  return s - bf16_to_f32(c);
}

void orc_compress_ef(const float* g, uint16_t* c, uint16_t* q, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float s = g[i] + ef_residual(c[i], q[i]);
    uint32_t w = enc_signed_bits(f2u(s));
    c[i] = (uint16_t)(w >> 16);
    q[i] = (uint16_t)(w & 0xFFFFu);
  }
}

/* value the residual field carries, for inspection */
void orc_ef_residual(const uint16_t* c, const uint16_t* q, float* e, int64_t n) {
  for (int64_t i = 0; i < n; ++i) e[i] = ef_residual(c[i], q[i]);
}

/* ---- per-tensor gradient statistics ---- */
void orc_grad_stats(const float* g, int64_t n, double* sumsq, float* amax, int64_t* nonfinite) {
  double s = 0.0;
  float a = 0.0f;
  int64_t bad = 0;
  for (int64_t i = 0; i < n; ++i) {
    float x = g[i];
    s += (double)x * (double)x;
    a = fmaxf(a, fabsf(x));
    if (!isfinite(x)) ++bad;
  }
  *sumsq = s;
  *amax = a;
  *nonfinite = bad;
}

/* ---- sign-fiber bit I/O over a list of second-moment tensors ---- */
void orc_fiber_read_bits(const uint32_t* words, int64_t n, uint8_t* bits) {
  for (int64_t i = 0; i < n; ++i) bits[i] = (uint8_t)(words[i] >> 31);
}
