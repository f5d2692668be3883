/*
 * hlkv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference HL-KV algorithms for the quantized KV-block
 * path.  It is the oracle that the CUDA kernels are compared against, and the
 * "port" CPU baseline of bench.py.  Nothing in the product library links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py do.
 *
 * Parity of this restatement is pinned two ways (tests/test_oracle_*.py):
 *   - the known-answer vectors of the reference's own tests
 *     (tests/project2/test_dequant.cpp, test_quant_encode.cpp,
 *      test_dequant_cuda.cpp, tests/project1/test_block_descriptor.cpp);
 *   - the reference library itself, compiled from its sources by
 *     oracle/build.py, and the fixtures in tests/golden/ generated from it.
 *
 * Every function names the reference lines it restates.  Compile with
 * -ffp-contract=off and without -ffast-math: binary32 arithmetic must round
 * exactly once per operation, as in the reference build.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ---- status codes: project2_quant/include/hl_quant/quant_types.hpp:54-60 ---------------- */
enum { ORC_OK = 0, ORC_INVALID_ARGUMENT = 1, ORC_BUFFER_TOO_SMALL = 2, ORC_UNSUPPORTED_FORMAT = 3 };

/* ---- format codes: quant_types.hpp:40-46 ------------------------------------------------ */
enum { F_FP16 = 0, F_E4M3 = 1, F_E5M2 = 2, F_INT4 = 3, F_INVALID = 15 };

/* Largest element count the reference accepts: SIZE_MAX / 2 (quant_types.hpp:105). */
#define ORC_MAX_ELEMENTS (SIZE_MAX / 2)

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---- minifloat bit specifications: project2_quant/src/minifloat_spec.hpp:11-24 ------------ */
typedef struct {
  uint32_t ebits, mbits;
  int32_t bias;
  int ieee_special;   /* all-ones exponent holds Inf/NaN (FP16, E5M2) */
  int saturating;     /* encode: overflow and +-Inf go to +-max (else to Inf) */
  uint32_t max_code;  /* magnitude code of the largest finite value */
  uint32_t nan_code;  /* magnitude code written for NaN */
  uint32_t inf_code;  /* magnitude code of Inf (ieee_special only) */
} mf_spec;

static const mf_spec kSpecFp16 = {5, 10, 15, 1, 0, 0x7BFFu, 0x7E00u, 0x7C00u};
static const mf_spec kSpecE4M3 = {4, 3, 7, 0, 1, 0x7Eu, 0x7Fu, 0u};
static const mf_spec kSpecE5M2 = {5, 2, 15, 1, 1, 0x7Bu, 0x7Fu, 0x7Cu};

/*
 * binary32 -> minifloat, round to nearest, ties to even, integer arithmetic.
 * Restates project2_quant/src/cpu_quant.cpp:27-64: the input is an integer
 * significand times a power of two; it is shifted down to the spacing of the
 * target at the input's binade (clamped below at the target's smallest normal
 * exponent, which makes subnormal targets fall out of the same formula) with
 * round-half-even on the dropped bits, and a carry out of the significand
 * moves into the exponent field by plain addition.
 */
static uint32_t mf_encode(float x, const mf_spec* s) {
  const uint32_t bits = f2u(x);
  const uint32_t sign = (bits >> 31) << (s->ebits + s->mbits);
  const uint32_t mag = bits & 0x7FFFFFFFu;
  const uint32_t overflow_code = s->saturating ? s->max_code : s->inf_code;
  if (mag > 0x7F800000u) return sign | s->nan_code;
  if (mag == 0x7F800000u) return sign | overflow_code;

  const int32_t emin = 1 - s->bias;
  int32_t binade;   /* unbiased exponent of the input, clamped at emin */
  int32_t lsb_exp;  /* exponent of bit 0 of `sig` */
  uint64_t sig;
  if (mag >= 0x00800000u) {
    const int32_t e = (int32_t)(mag >> 23) - 127;
    sig = (uint64_t)((mag & 0x007FFFFFu) | 0x00800000u);
    lsb_exp = e - 23;
    binade = e < emin ? emin : e;
  } else { /* binary32 subnormal or zero: below every target's emin */
    sig = mag;
    lsb_exp = -149;
    binade = emin;
  }
  const int32_t drop = (binade - (int32_t)s->mbits) - lsb_exp; /* >= 1 since mbits < 23 */
  uint64_t kept = 0;
  if (drop < 40) { /* otherwise the value is below 2^-16 of one target spacing: rounds to 0 */
    const uint32_t d = (uint32_t)drop;
    kept = sig >> d;
    const uint64_t rest = sig & ((1ull << d) - 1ull);
    const uint64_t half = 1ull << (d - 1);
    if (rest > half || (rest == half && (kept & 1ull))) kept += 1ull;
  }
  const uint64_t code = ((uint64_t)(binade - emin) << s->mbits) + kept;
  if (code > s->max_code) return sign | overflow_code;
  return sign | (uint32_t)code;
}

/*
 * minifloat -> binary32, exact.  Same results as project2_quant/src/cpu_dequant.cpp:20-47;
 * normals are built from bits, subnormals as (integer mantissa) * 2^(1-bias-mbits),
 * a product of two exactly representable binary32 values whose result is a
 * binary32 normal, hence exact.
 */
static float mf_decode(uint32_t code, const mf_spec* s) {
  const uint32_t width = s->ebits + s->mbits;
  const uint32_t sbit = ((code >> width) & 1u) << 31;
  const uint32_t mag = code & ((1u << width) - 1u);
  const uint32_t ef = mag >> s->mbits;
  const uint32_t mf = mag & ((1u << s->mbits) - 1u);
  const uint32_t e_all = (1u << s->ebits) - 1u;
  if (s->ieee_special && ef == e_all) return u2f(sbit | (mf == 0 ? 0x7F800000u : 0x7FC00000u));
  if (!s->ieee_special && mag > s->max_code) return u2f(sbit | 0x7FC00000u); /* E4M3FN S.1111.111 */
  if (ef == 0) {
    if (mf == 0) return u2f(sbit);
    const float unit = u2f((uint32_t)(1 - s->bias - (int32_t)s->mbits + 127) << 23);
    const float v = (float)mf * unit;
    return u2f(sbit | f2u(v));
  }
  return u2f(sbit | ((uint32_t)((int32_t)ef - s->bias + 127) << 23) | (mf << (23 - s->mbits)));
}

ORC_API uint16_t orc_encode_fp16(float x) { return (uint16_t)mf_encode(x, &kSpecFp16); }
ORC_API uint8_t orc_encode_e4m3(float x) { return (uint8_t)mf_encode(x, &kSpecE4M3); }
ORC_API uint8_t orc_encode_e5m2(float x) { return (uint8_t)mf_encode(x, &kSpecE5M2); }
ORC_API float orc_decode_fp16(uint16_t c) { return mf_decode(c, &kSpecFp16); }
ORC_API float orc_decode_e4m3(uint8_t c) { return mf_decode(c, &kSpecE4M3); }
ORC_API float orc_decode_e5m2(uint8_t c) { return mf_decode(c, &kSpecE5M2); }

/* Array forms, for exhaustive and bulk comparisons from Python. */
ORC_API void orc_encode_array(int format, const float* in, size_t n, uint16_t* out) {
  const mf_spec* s = format == F_FP16 ? &kSpecFp16 : format == F_E4M3 ? &kSpecE4M3 : &kSpecE5M2;
  for (size_t i = 0; i < n; ++i) out[i] = (uint16_t)mf_encode(in[i], s);
}
ORC_API void orc_decode_array(int format, const uint16_t* in, size_t n, float* out) {
  const mf_spec* s = format == F_FP16 ? &kSpecFp16 : format == F_E4M3 ? &kSpecE4M3 : &kSpecE5M2;
  for (size_t i = 0; i < n; ++i) out[i] = mf_decode(in[i], s);
}

/* ---- format rules: quant_types.hpp:90-132 ----------------------------------------------- */
static int fmt_valid(int f) { return f >= 0 && f <= 3; }
static int fmt_uses_params(int f) { return f != F_FP16; }
static size_t fmt_packed_bytes(int f, size_t n) {
  if (f == F_FP16) return 2 * n;
  if (f == F_INT4) return n / 2 + (n % 2);
  return n;
}
static size_t num_groups(size_t n, size_t g) { return g == 0 ? 0 : n / g + (n % g != 0); }
static int group_ok(int f, size_t g) {
  if (!fmt_uses_params(f)) return g == 0;
  return g > 0 && (f != F_INT4 || g % 2 == 0);
}

/* ---- element access: cpu_quant.cpp:66-81 (write_code), cpu_dequant.cpp:49-61 (read_code) - */
static void put_code(int f, uint8_t* p, size_t i, uint32_t code) {
  switch (f) {
    case F_FP16: p[2 * i] = (uint8_t)code; p[2 * i + 1] = (uint8_t)(code >> 8); break;
    case F_E4M3: case F_E5M2: p[i] = (uint8_t)code; break;
    default: p[i / 2] |= (uint8_t)((code & 0xFu) << (4 * (i % 2))); break;
  }
}
static uint32_t get_code(int f, const uint8_t* p, size_t i) {
  switch (f) {
    case F_FP16: return (uint32_t)p[2 * i] | ((uint32_t)p[2 * i + 1] << 8);
    case F_E4M3: case F_E5M2: return p[i];
    default: return (p[i / 2] >> (4 * (i % 2))) & 0xFu;
  }
}

/*
 * quantize_reference, project2_quant/src/cpu_quant.cpp:97-170.  Parameters are
 * 2 floats per group {scale, bias} (AffineParams, quant_types.hpp:65-69).
 * Everything is validated before anything is written.
 */
ORC_API int orc_quantize(int f, const float* in, size_t n, size_t g, float* params,
                         size_t n_params, uint8_t* packed, size_t packed_size) {
  if (!fmt_valid(f)) return ORC_UNSUPPORTED_FORMAT;
  if (n > ORC_MAX_ELEMENTS) return ORC_INVALID_ARGUMENT;
  if (!group_ok(f, g)) return ORC_INVALID_ARGUMENT;
  const size_t groups = num_groups(n, g);
  if (n_params != groups) return ORC_INVALID_ARGUMENT;
  if (fmt_uses_params(f)) {
    for (size_t i = 0; i < n; ++i)
      if (!isfinite(in[i])) return ORC_INVALID_ARGUMENT;
    if (f == F_INT4) {
      for (size_t k = 0; k < groups; ++k) {
        const size_t b = k * g, e = (k + 1) * g < n ? (k + 1) * g : n;
        float lo = in[b], hi = in[b];
        for (size_t i = b; i < e; ++i) {
          if (in[i] < lo) lo = in[i];
          if (!(in[i] < hi)) hi = in[i];
        }
        if (!isfinite(hi - lo)) return ORC_INVALID_ARGUMENT;
      }
    }
  }
  const size_t bytes = fmt_packed_bytes(f, n);
  if (packed_size < bytes) return ORC_BUFFER_TOO_SMALL;
  memset(packed, 0, bytes);

  if (f == F_FP16) {
    for (size_t i = 0; i < n; ++i) put_code(f, packed, i, mf_encode(in[i], &kSpecFp16));
    return ORC_OK;
  }
  for (size_t k = 0; k < groups; ++k) {
    const size_t b = k * g, e = (k + 1) * g < n ? (k + 1) * g : n;
    if (f == F_E4M3 || f == F_E5M2) { /* cpu_quant.cpp:138-150 */
      const mf_spec* s = f == F_E4M3 ? &kSpecE4M3 : &kSpecE5M2;
      const float max_finite = f == F_E4M3 ? 448.0f : 57344.0f;
      float amax = 0.0f;
      for (size_t i = b; i < e; ++i) {
        const float a = fabsf(in[i]);
        if (amax < a) amax = a;
      }
      float scale = 1.0f;
      if (amax > 0.0f) {
        const float q = amax / max_finite;
        const float tiny = u2f(0x00800000u); /* FLT_MIN */
        scale = q < tiny ? tiny : q;
      }
      params[2 * k] = scale;
      params[2 * k + 1] = 0.0f;
      for (size_t i = b; i < e; ++i) put_code(f, packed, i, mf_encode(in[i] / scale, s));
    } else { /* INT4, cpu_quant.cpp:151-166: first minimum, last maximum (std::minmax_element) */
      float lo = in[b], hi = in[b];
      for (size_t i = b; i < e; ++i) {
        if (in[i] < lo) lo = in[i];
        if (!(in[i] < hi)) hi = in[i];
      }
      const float scale = (hi - lo) / 15.0f;
      params[2 * k] = scale;
      params[2 * k + 1] = lo;
      for (size_t i = b; i < e; ++i) {
        uint32_t q = 0;
        if (scale > 0.0f) {
          const float r = nearbyintf((in[i] - lo) / scale);
          const float c = r < 0.0f ? 0.0f : (15.0f < r ? 15.0f : r);
          q = (uint32_t)c;
        }
        put_code(f, packed, i, q);
      }
    }
  }
  return ORC_OK;
}

/* check_args, project2_quant/src/cpu_dequant.cpp:77-90. */
static int dq_check(int f, size_t packed_size, size_t n, const float* params, size_t n_params,
                    size_t g) {
  if (!fmt_valid(f)) return ORC_UNSUPPORTED_FORMAT;
  if (n > ORC_MAX_ELEMENTS) return ORC_INVALID_ARGUMENT;
  if (!group_ok(f, g)) return ORC_INVALID_ARGUMENT;
  if (n_params != num_groups(n, g)) return ORC_INVALID_ARGUMENT;
  for (size_t k = 0; k < n_params; ++k) {
    if (!isfinite(params[2 * k]) || !isfinite(params[2 * k + 1])) return ORC_INVALID_ARGUMENT;
    if (f != F_INT4 && params[2 * k + 1] != 0.0f) return ORC_INVALID_ARGUMENT;
  }
  if (packed_size < fmt_packed_bytes(f, n)) return ORC_BUFFER_TOO_SMALL;
  return ORC_OK;
}

/* reference_value, project2_quant/src/cpu_dequant.cpp:93-109. */
static float dq_value(int f, const uint8_t* packed, size_t i, const float* params, size_t g) {
  const uint32_t c = get_code(f, packed, i);
  switch (f) {
    case F_FP16: return mf_decode(c, &kSpecFp16);
    case F_E4M3: return mf_decode(c, &kSpecE4M3) * params[2 * (i / g)];
    case F_E5M2: return mf_decode(c, &kSpecE5M2) * params[2 * (i / g)];
    default: return fmaf((float)c, params[2 * (i / g)], params[2 * (i / g) + 1]);
  }
}

/* dequantize_reference, cpu_dequant.cpp:113-125. */
ORC_API int orc_dequantize(int f, const uint8_t* packed, size_t packed_size, size_t n,
                           const float* params, size_t n_params, size_t g, float* out,
                           size_t out_size) {
  const int st = dq_check(f, packed_size, n, params, n_params, g);
  if (st != ORC_OK) return st;
  if (out_size < n) return ORC_BUFFER_TOO_SMALL;
  for (size_t i = 0; i < n; ++i) out[i] = dq_value(f, packed, i, params, g);
  return ORC_OK;
}

/*
 * dequantize_reference_to_fp16, cpu_dequant.cpp:127-141: the binary32 value of
 * dequantize_reference rounded to binary16 with encode_fp16.  On x86-64 (SSE),
 * a product with a NaN operand returns that NaN and Inf*0 returns the default
 * NaN, whose sign bit is set; encode_fp16 keeps the sign, so those become
 * sign|0x7E00 and 0xFE00.  The CUDA kernels reproduce exactly these bits.
 */
ORC_API int orc_dequantize_to_fp16(int f, const uint8_t* packed, size_t packed_size, size_t n,
                                   const float* params, size_t n_params, size_t g, uint16_t* out,
                                   size_t out_size) {
  const int st = dq_check(f, packed_size, n, params, n_params, g);
  if (st != ORC_OK) return st;
  if (out_size < n) return ORC_BUFFER_TOO_SMALL;
  for (size_t i = 0; i < n; ++i)
    out[i] = (uint16_t)mf_encode(dq_value(f, packed, i, params, g), &kSpecFp16);
  return ORC_OK;
}

/* ==== the heterogeneous block path ======================================================== */
/*
 * Block payload layout (the layout tag stored in BlockExecDescriptor::info
 * bits 6..9, block_descriptor.hpp:137-145): a block holds 2 (K,V) x T tokens x H
 * heads rows of D elements, row-major in that order; one parameter group per
 * row.  The slot holds packed_bytes(format, rows*D) bytes of codes followed by
 * the parameters: nothing for FP16, one binary32 scale per row for FP8, one
 * {scale, bias} pair per row for INT4.  Rows of tokens >= valid_tokens are
 * written as +0.
 *
 * The device descriptor table is 4 uint32 words per block id:
 * {slot, info, scale_ref, block_id} (block_descriptor.hpp:146-150); the arena is
 * uint32 block ids; a segment is {offset, length} (id_arena.hpp:39-43).
 */
typedef struct {
  const uint8_t* base;
  uint64_t slot_bytes;
  uint32_t num_slots;
  uint32_t pad;
} orc_pool;

/* Error bits; identical to the HLKV_ERR_* values of include/hlkv.h. */
enum {
  E_NOT_EXECUTABLE = 1u << 0,
  E_BAD_FORMAT = 1u << 1,
  E_SLOT_RANGE = 1u << 2,
  E_ARENA_RANGE = 1u << 3,
  E_BLOCK_ID_RANGE = 1u << 4,
  E_VALID_TOKENS = 1u << 5,
  E_LAYOUT = 1u << 6,
  E_SCALE_MODE = 1u << 7,
  E_DESC_MISMATCH = 1u << 8,
  E_NONFINITE = 1u << 9,
  E_TOKEN_RANGE = 1u << 10,
  E_PATCH_RANGE = 1u << 11,
  E_OUT_ALIGN = 1u << 12,
};

typedef struct {
  uint32_t T, H, D, layout_id;
} orc_geom;

static size_t slot_need(int f, const orc_geom* g) {
  const size_t elems = (size_t)2 * g->T * g->H * g->D, rows = (size_t)2 * g->T * g->H;
  if (f == F_FP16) return 2 * elems;
  if (f == F_INT4) return elems / 2 + 8 * rows;
  return elems + 4 * rows;
}

/*
 * The dequantization parameters {scale, bias} of row r of a quantized block, by the
 * descriptor's scale_mode (ScaleMode, block_descriptor.hpp:61-72):
 *   0 kNone: per row, stored after the codes (FP8: binary32 scale; INT4: scale, bias);
 *   1 kInlineF32: one scale for the whole block, the binary32 bits of scale_ref
 *     (BlockExecDescriptor::inline_scale_f32, block_descriptor.hpp:179-182), bias 0;
 *   2 kInlineF16Pair: binary16 scale in bits 0..15 and bias in bits 16..31 of scale_ref
 *     (hl_allocator_abi.md:62), widened exactly.
 * With a block-wide mode the block is one group of dequantize_reference_to_fp16
 * (cpu_dequant.cpp:127-141) with these parameters; FP8 decoding reads the scale only.
 */
static void row_params(int f, uint32_t mode, uint32_t scale_ref, const uint8_t* payload,
                       size_t code_bytes, size_t r, float p[2]) {
  p[0] = 0.0f;
  p[1] = 0.0f;
  if (mode == 1) {
    memcpy(&p[0], &scale_ref, 4);
  } else if (mode == 2) {
    p[0] = mf_decode(scale_ref & 0xFFFFu, &kSpecFp16);
    p[1] = mf_decode(scale_ref >> 16, &kSpecFp16);
  } else if (f == F_E4M3 || f == F_E5M2) {
    memcpy(&p[0], payload + code_bytes + 4 * r, 4);
  } else if (f == F_INT4) {
    memcpy(p, payload + code_bytes + 8 * r, 8);
  }
}

/*
 * Resolves block j of a segment to its payload, or returns the first failing
 * check as an error bit (0 = ok).  Check order is part of the contract: the
 * kernels report the same single bit per block.  Quantized blocks may carry
 * block-wide parameters (scale modes 1 and 2); scale mode 3 (kExternal, an index
 * into a scale pool the ABI does not pass) is rejected.
 */
static uint32_t resolve_block(const orc_pool* pools, const orc_geom* g, const uint32_t* table,
                              uint32_t table_size, const uint32_t* arena, uint32_t arena_size,
                              uint64_t arena_pos, int* fmt, const uint8_t** payload,
                              uint32_t* valid, uint32_t* scale_mode, uint32_t* scale_ref) {
  if (arena_pos >= arena_size) return E_ARENA_RANGE;
  const uint32_t id = arena[arena_pos];
  if (id >= table_size) return E_BLOCK_ID_RANGE;
  const uint32_t* d = table + 4 * (size_t)id;
  const uint32_t slot = d[0], info = d[1], bid = d[3];
  if (bid != id) return E_DESC_MISMATCH;
  const uint32_t f = info & 0xFu, mode = (info >> 4) & 3u, layout = (info >> 6) & 0xFu,
                 vt = (info >> 10) & 0x3FFu;
  if (f == F_INVALID) return E_NOT_EXECUTABLE;
  if (f > 3 || pools[f].base == NULL || pools[f].num_slots == 0) return E_BAD_FORMAT;
  if (layout != g->layout_id) return E_LAYOUT;
  if (f != F_FP16 && mode > 2) return E_SCALE_MODE;
  if (f != F_FP16 && mode != 0) {
    /* Block-wide parameters must be what dequantize_reference accepts
       (cpu_dequant.hpp:33, cpu_dequant.cpp:85): finite scale and bias, FP8 bias 0. */
    float p[2];
    row_params((int)f, mode, d[2], NULL, 0, 0, p);
    if (!isfinite(p[0]) || !isfinite(p[1]) || (f != F_INT4 && p[1] != 0.0f)) return E_SCALE_MODE;
  }
  if (vt > g->T) return E_VALID_TOKENS;
  if (slot >= pools[f].num_slots) return E_SLOT_RANGE;
  *fmt = (int)f;
  *payload = pools[f].base + (size_t)slot * pools[f].slot_bytes;
  *valid = vt;
  *scale_mode = f == F_FP16 ? 0u : mode;
  *scale_ref = d[2];
  return 0;
}

/* Decodes one resolved block into out[0 .. 2*T*H*D). */
static void decode_block(int f, const uint8_t* payload, uint32_t vt, uint32_t mode,
                         uint32_t scale_ref, const orc_geom* g, uint16_t* out) {
  const size_t rows = (size_t)2 * g->T * g->H, D = g->D, rows_per_kv = (size_t)g->T * g->H;
  const size_t code_bytes = fmt_packed_bytes(f, rows * D);
  for (size_t r = 0; r < rows; ++r) {
    const size_t r_in_kv = r < rows_per_kv ? r : r - rows_per_kv;
    uint16_t* o = out + r * D;
    if (r_in_kv >= (size_t)vt * g->H) {
      memset(o, 0, 2 * D);
      continue;
    }
    float p[2];
    const uint8_t* codes = payload + fmt_packed_bytes(f, r * D);
    row_params(f, mode, scale_ref, payload, code_bytes, r, p);
    /* One group per row, or one per block with the same parameters in every row:
       dequantize_reference_to_fp16 on D elements. */
    for (size_t i = 0; i < D; ++i)
      o[i] = (uint16_t)mf_encode(dq_value(f, codes, i, p, D), &kSpecFp16);
  }
}

typedef struct {
  const orc_pool* pools;
  const orc_geom* g;
  const uint32_t* table;
  uint32_t table_size;
  const uint32_t* arena;
  uint32_t arena_size;
  const uint32_t* segs;
  uint32_t nseq;
  const uint64_t* out_offsets;
  uint16_t* out;
  const uint64_t* prefix; /* blocks before sequence i */
  uint64_t item_begin, item_end;
  uint32_t err;
} gather_job;

static void* gather_worker(void* arg) {
  gather_job* jb = (gather_job*)arg;
  const size_t belems = (size_t)2 * jb->g->T * jb->g->H * jb->g->D;
  uint32_t seq = 0;
  for (uint64_t w = jb->item_begin; w < jb->item_end; ++w) {
    while (seq + 1 < jb->nseq && jb->prefix[seq + 1] <= w) ++seq;
    const uint64_t j = w - jb->prefix[seq];
    const uint64_t base = jb->out_offsets ? jb->out_offsets[seq] : jb->prefix[seq] * belems;
    if (base % 8 != 0) { jb->err |= E_OUT_ALIGN; continue; }
    int f = 0;
    const uint8_t* payload = NULL;
    uint32_t vt = 0, mode = 0, sref = 0;
    const uint32_t e = resolve_block(jb->pools, jb->g, jb->table, jb->table_size, jb->arena,
                                     jb->arena_size, (uint64_t)jb->segs[2 * seq] + j, &f,
                                     &payload, &vt, &mode, &sref);
    if (e) { jb->err |= e; continue; }
    decode_block(f, payload, vt, mode, sref, jb->g, jb->out + base + j * belems);
  }
  return NULL;
}

/*
 * Gather-dequant oracle: block j of sequence i is
 *   table[arena[segs[i].offset + j]]   (hetero_block_table.hpp:22-25)
 * and lands at out[out_offsets[i] + j*block_elems] (packed when out_offsets is
 * NULL).  Blocks that fail a check are skipped (output untouched) and their
 * error bit is OR-ed into the return value.  `threads` > 1 splits the blocks
 * over POSIX threads (the CPU baseline); the result does not depend on it.
 */
ORC_API uint32_t orc_gather_dequant(const orc_pool* pools, uint32_t T, uint32_t H, uint32_t D,
                                    uint32_t layout_id, const uint32_t* table,
                                    uint32_t table_size, const uint32_t* arena,
                                    uint32_t arena_size, const uint32_t* segs, uint32_t nseq,
                                    const uint64_t* out_offsets, uint16_t* out,
                                    const uint64_t* prefix, int threads) {
  const orc_geom g = {T, H, D, layout_id};
  if (nseq == 0) return 0;
  const uint64_t total = prefix[nseq];
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  gather_job jobs[256];
  pthread_t tids[256];
  for (int t = 0; t < threads; ++t) {
    gather_job* jb = &jobs[t];
    jb->pools = pools; jb->g = &g; jb->table = table; jb->table_size = table_size;
    jb->arena = arena; jb->arena_size = arena_size; jb->segs = segs; jb->nseq = nseq;
    jb->out_offsets = out_offsets; jb->out = out; jb->prefix = prefix;
    jb->item_begin = total * (uint64_t)t / (uint64_t)threads;
    jb->item_end = total * (uint64_t)(t + 1) / (uint64_t)threads;
    jb->err = 0;
  }
  if (threads == 1) {
    gather_worker(&jobs[0]);
  } else {
    for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, gather_worker, &jobs[t]);
    for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
  }
  uint32_t err = 0;
  for (int t = 0; t < threads; ++t) err |= jobs[t].err;
  return err;
}

/*
 * Delta apply oracle: the device-side restatement of ExecMirror::apply
 * (tests/project1/exec_mirror.hpp:23-49) after growth, i.e. the protocol of
 * ExecDelta (hetero_block_table.hpp:100-114):
 *   table[p.block_id] = p  for every 16-byte descriptor patch,
 *   arena[p.offset] = p.block_id  for every {offset, block_id} id patch.
 * Out-of-range targets are skipped and reported with E_PATCH_RANGE.
 */
ORC_API uint32_t orc_apply_delta(uint32_t* table, uint32_t table_size, uint32_t* arena,
                                 uint32_t arena_size, const uint32_t* desc_patches, uint32_t n_desc,
                                 const uint32_t* id_patches, uint32_t n_id) {
  uint32_t err = 0;
  for (uint32_t k = 0; k < n_desc; ++k) {
    const uint32_t* p = desc_patches + 4 * (size_t)k;
    if (p[3] >= table_size) { err |= E_PATCH_RANGE; continue; }
    memcpy(table + 4 * (size_t)p[3], p, 16);
  }
  for (uint32_t k = 0; k < n_id; ++k) {
    const uint32_t off = id_patches[2 * (size_t)k], id = id_patches[2 * (size_t)k + 1];
    if (off >= arena_size) { err |= E_PATCH_RANGE; continue; }
    arena[off] = id;
  }
  return err;
}

/*
 * Append-encode oracle: token k (FP16, rows [kv][head] of D elements, so
 * 2*H*D values) is written into token slot targets[k].token of block
 * targets[k].block_id, through the device descriptor table.  Each row is one
 * group of quantize_reference (cpu_quant.cpp:97-170) on the binary32 values
 * of the FP16 inputs; the codes go to row (kv*T + token)*H + h of the block,
 * the parameters to the same row of the parameter area.  A target that fails
 * a check is skipped; a row with a non-finite input (FP8/INT4) is skipped
 * with E_NONFINITE, which is where quantize_reference returns kInvalidArgument.
 */
ORC_API uint32_t orc_append_encode(const orc_pool* pools, uint32_t T, uint32_t H, uint32_t D,
                                   uint32_t layout_id, const uint32_t* table,
                                   uint32_t table_size, const uint32_t* targets, uint32_t n,
                                   const uint16_t* tokens) {
  uint32_t err = 0;
  float vals[4096];
  uint8_t codes[8192];
  if (D > 4096) return E_LAYOUT;
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t id = targets[2 * (size_t)k], tok = targets[2 * (size_t)k + 1];
    if (id >= table_size) { err |= E_BLOCK_ID_RANGE; continue; }
    const uint32_t* d = table + 4 * (size_t)id;
    const uint32_t slot = d[0], info = d[1];
    const uint32_t f = info & 0xFu, mode = (info >> 4) & 3u, layout = (info >> 6) & 0xFu;
    if (d[3] != id) { err |= E_DESC_MISMATCH; continue; }
    if (f == F_INVALID) { err |= E_NOT_EXECUTABLE; continue; }
    if (f > 3 || pools[f].base == NULL || pools[f].num_slots == 0) { err |= E_BAD_FORMAT; continue; }
    if (layout != layout_id) { err |= E_LAYOUT; continue; }
    if (f != F_FP16 && mode != 0) { err |= E_SCALE_MODE; continue; }
    if (tok >= T) { err |= E_TOKEN_RANGE; continue; }
    if (slot >= pools[f].num_slots) { err |= E_SLOT_RANGE; continue; }
    uint8_t* payload = (uint8_t*)pools[f].base + (size_t)slot * pools[f].slot_bytes;
    const size_t rows = (size_t)2 * T * H;
    const size_t code_bytes = fmt_packed_bytes((int)f, rows * D);
    for (uint32_t kv = 0; kv < 2; ++kv) {
      for (uint32_t h = 0; h < H; ++h) {
        const uint16_t* src = tokens + ((size_t)k * 2 * H + (size_t)kv * H + h) * D;
        const size_t row = ((size_t)kv * T + tok) * H + h;
        for (uint32_t i = 0; i < D; ++i) vals[i] = mf_decode(src[i], &kSpecFp16);
        float p[2];
        const size_t nb = fmt_packed_bytes((int)f, D);
        const int st = orc_quantize((int)f, vals, D, f == F_FP16 ? 0 : D, p,
                                    f == F_FP16 ? 0 : 1, codes, sizeof(codes));
        if (st != ORC_OK) { err |= E_NONFINITE; continue; }
        memcpy(payload + fmt_packed_bytes((int)f, row * D), codes, nb);
        if (f == F_E4M3 || f == F_E5M2) memcpy(payload + code_bytes + 4 * row, &p[0], 4);
        if (f == F_INT4) memcpy(payload + code_bytes + 8 * row, p, 8);
      }
    }
  }
  return err;
}

/* ---- format-change transcode (device half of hetero_block_table.cpp:251-287) ---------------- */
/* Job k: {from_format, from_slot, to_format, to_slot, valid_tokens, from_scale_mode,
 * from_scale_ref, 0}.  Each row of a valid token is decoded with dequantize_reference_to_fp16
 * (cpu_dequant.cpp:127-141) from the source slot, with the source block's parameters
 * (row_params: per row, or block-wide by its scale mode; mode 3 is rejected) and re-encoded with quantize_reference (cpu_quant.cpp:97-170) on the binary32
 * values of those binary16 results into the destination slot; rows of later tokens are
 * encoded from +0.  A rejected row leaves the destination row untouched (E_NONFINITE). */
ORC_API uint32_t orc_transcode(const orc_pool* pools, uint32_t T, uint32_t H, uint32_t D,
                               const uint32_t* jobs, uint32_t n) {
  uint32_t err = 0;
  float vals[4096];
  uint16_t half[4096];
  uint8_t codes[8192];
  if (D > 4096) return E_LAYOUT;
  const size_t rows = (size_t)2 * T * H;
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t* j = jobs + 8 * (size_t)k;
    const uint32_t ff = j[0], fs = j[1], tf = j[2], ts = j[3], vt = j[4];
    const uint32_t fmode = ff == F_FP16 ? 0u : j[5], fref = j[6]; /* the source's scale mode */
    if (ff > 3 || tf > 3 || pools[ff].base == NULL || pools[tf].base == NULL) { err |= E_BAD_FORMAT; continue; }
    if (fmode > 2) { err |= E_SCALE_MODE; continue; }
    if (fmode != 0) {
      float q[2];
      row_params((int)ff, fmode, fref, NULL, 0, 0, q);
      if (!isfinite(q[0]) || !isfinite(q[1]) || (ff != F_INT4 && q[1] != 0.0f)) { err |= E_SCALE_MODE; continue; }
    }
    if (fs >= pools[ff].num_slots || ts >= pools[tf].num_slots) { err |= E_SLOT_RANGE; continue; }
    if (vt > T) { err |= E_VALID_TOKENS; continue; }
    const uint8_t* src = pools[ff].base + (size_t)fs * pools[ff].slot_bytes;
    uint8_t* dst = (uint8_t*)pools[tf].base + (size_t)ts * pools[tf].slot_bytes;
    const size_t src_codes = fmt_packed_bytes((int)ff, rows * D);
    const size_t dst_codes = fmt_packed_bytes((int)tf, rows * D);
    for (size_t r = 0; r < rows; ++r) {
      const uint32_t tok = (uint32_t)((r / H) % T);
      if (tok < vt) {
        float p[2];
        row_params((int)ff, fmode, fref, src, src_codes, r, p);
        const int st = orc_dequantize_to_fp16((int)ff, src + fmt_packed_bytes((int)ff, r * D),
                                              fmt_packed_bytes((int)ff, D), D, p,
                                              ff == F_FP16 ? 0 : 1, ff == F_FP16 ? 0 : D, half, D);
        if (st != ORC_OK) { err |= E_NONFINITE; continue; }
        for (uint32_t i = 0; i < D; ++i) vals[i] = mf_decode(half[i], &kSpecFp16);
      } else {
        for (uint32_t i = 0; i < D; ++i) vals[i] = 0.0f;
      }
      float p[2];
      const int st = orc_quantize((int)tf, vals, D, tf == F_FP16 ? 0 : D, p, tf == F_FP16 ? 0 : 1,
                                  codes, sizeof(codes));
      if (st != ORC_OK) { err |= E_NONFINITE; continue; }
      memcpy(dst + fmt_packed_bytes((int)tf, r * D), codes, fmt_packed_bytes((int)tf, D));
      if (tf == F_E4M3 || tf == F_E5M2) memcpy(dst + dst_codes + 4 * r, &p[0], 4);
      if (tf == F_INT4) memcpy(dst + dst_codes + 8 * r, p, 8);
    }
  }
  return err;
}

ORC_API size_t orc_slot_bytes_needed(int f, uint32_t T, uint32_t H, uint32_t D) {
  const orc_geom g = {T, H, D, 1};
  return slot_need(f, &g);
}

/* ---- seeded synthetic data: tests/project2/test_dequant.cpp:180-202 ---------------------- */
/* SplitMix64 and Box-Muller, as the reference tests generate N(0,1) data. */
ORC_API void orc_gaussian(uint64_t seed, float sigma, float* out, size_t n) {
  uint64_t st = seed;
  for (size_t i = 0; i < n; ++i) {
    uint64_t z;
    z = (st += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const double u1 = 1.0 - (double)(z >> 11) * 0x1.0p-53;
    z = (st += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const double u2 = (double)(z >> 11) * 0x1.0p-53;
    out[i] = sigma * (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
  }
}

/* ---- per-row encode over threads (the decode-append CPU baseline) ------------------------- */
/* quantize_reference per row of D values (cpu_quant.cpp:97-170), one group per row, row r
 * in format fmt[r] (E4M3, E5M2 or INT4); codes of row r at codes + r * D, params {scale, bias}
 * at params + 2r.
 * Returns the number of rows rejected. */
typedef struct {
  const uint8_t* fmt;
  const float* in;
  size_t lo, hi, D, bad;
  float* params;
  uint8_t* codes;
} rows_job;

static void* rows_worker(void* arg) {
  rows_job* j = (rows_job*)arg;
  for (size_t r = j->lo; r < j->hi; ++r) {
    if (orc_quantize((int)j->fmt[r], j->in + r * j->D, j->D, j->D, j->params + 2 * r, 1,
                     j->codes + r * j->D, j->D) != ORC_OK) {
      ++j->bad;
    }
  }
  return NULL;
}

ORC_API size_t orc_quantize_rows(const uint8_t* fmt, const float* in, size_t rows, size_t D,
                                 float* params, uint8_t* codes, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tids[256];
  rows_job jobs[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (rows_job){fmt, in, rows * (size_t)t / (size_t)threads,
                         rows * (size_t)(t + 1) / (size_t)threads, D, 0, params, codes};
    pthread_create(&tids[t], NULL, rows_worker, &jobs[t]);
  }
  size_t bad = 0;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tids[t], NULL);
    bad += jobs[t].bad;
  }
  return bad;
}
