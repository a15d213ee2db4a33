/*
 * t5e_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-case-at-a-time restatement of the tcgen05_model arithmetic
 * (the reference Python package sf-tensor/tcgen05).  It is the parity reference
 * for the CUDA emulator and the timed CPU baseline ("port") in bench.py.  It is
 * never linked into, called by, or shipped with the product path.
 *
 * Every function follows one reference function and cites it as
 * path:line inside the reference project.  The reference computes with
 * unbounded Python integers; this restatement uses __int128 for every
 * accumulator and aborts (status ORACLE_ERR_RANGE) if a shift would leave the
 * range in which __int128 is exact, so a silent divergence is impossible.
 *
 * Parity of this file is pinned by tests/test_oracle_golden.py against the
 * reference's own frozen B200 words (tcgen05_model/validation.py:37-344,
 * tests/test_model.py:141-169) and against fixtures produced by running the
 * reference itself (tests/golden/make_golden.py).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <limits.h>

typedef __int128 i128;

/* ---- operand formats (names follow tcgen05_model.normalize_format) ---- */
enum {
    OF_TF32 = 0, OF_BF16 = 1, OF_F16 = 2, OF_E4M3 = 3, OF_E5M2 = 4,
    OF_E2M3 = 5, OF_E3M2 = 6, OF_E2M1 = 7, OF_U8 = 8, OF_S8 = 9,
    OF_NONE = -1
};
enum { OD_F32 = 0, OD_F16 = 1, OD_S32 = 2 };
enum { OS_NONE = 0, OS_UE8M0 = 1, OS_UE4M3 = 2 };
enum { OK_NONE = 0, OK_MXF8F6F4 = 1, OK_MXF4 = 2, OK_MXF4NVF4 = 3, OK_NVFP4 = 4 };

/* status codes: 0 ok, negative = the reference raises ValueError */
enum {
    ORACLE_OK = 0,
    ORACLE_ERR_DESCRIPTOR = -1,   /* make_model ValueError */
    ORACLE_ERR_KIND = -2,         /* sparse_active_indices kind ValueError */
    ORACLE_ERR_META_WORDS = -3,   /* too few metadata nibbles */
    ORACLE_ERR_SELECTOR = -4,     /* illegal sparse selector */
    ORACLE_ERR_EMPTY = -5,        /* empty dot product */
    ORACLE_ERR_SCALE_PAIR = -6,   /* scale_a/scale_b supplied alone */
    ORACLE_ERR_SCALE_COUNT = -7,  /* scale block counts differ */
    ORACLE_ERR_SCALE_COVER = -8,  /* more K than scale blocks cover */
    ORACLE_ERR_SCALE_VALUE = -9,  /* scale is not an 8-bit word */
    ORACLE_ERR_RANGE = -100       /* restatement left its exact range */
};

/* ---- decoded operand: tcgen05_model/model.py:72-239 return shape ---- */
enum { T_FIN = 0, T_NAN = 1, T_PINF = 2, T_NINF = 3 };
typedef struct { int tag; int64_t mant; int ve; int re; } dec_t;

static dec_t fin(int64_t mant, int ve, int re) { dec_t d = {T_FIN, mant, ve, re}; return d; }
static dec_t special(int tag) { dec_t d = {tag, 0, 0, 0}; return d; }

/* model.py:72-87 */
static dec_t dec_tf32(uint32_t bits) {
    bits &= 0xFFFFE000u;
    int sign = (bits & 0x80000000u) ? -1 : 1;
    int exp = (bits & 0x7F800000u) >> 23;
    uint32_t frac = bits & 0x007FFFFFu;
    if (exp == 0xFF) return frac ? special(T_NAN) : special(sign < 0 ? T_NINF : T_PINF);
    int64_t mant; int raw;
    if (exp == 0) { mant = frac >> 13; raw = 1 - 127; }
    else { mant = (1 << 10) | (frac >> 13); raw = exp - 127; }
    return fin(sign * mant, raw - 10, raw);
}

/* model.py:90-105 */
static dec_t dec_bf16(uint32_t bits) {
    bits &= 0xFFFF0000u;
    int sign = (bits & 0x80000000u) ? -1 : 1;
    int exp = (bits & 0x7F800000u) >> 23;
    uint32_t frac = bits & 0x007FFFFFu;
    if (exp == 0xFF) return frac ? special(T_NAN) : special(sign < 0 ? T_NINF : T_PINF);
    int64_t mant; int raw;
    if (exp == 0) { mant = frac >> 16; raw = 1 - 127; }
    else { mant = (1 << 7) | (frac >> 16); raw = exp - 127; }
    return fin(sign * mant, raw - 7, raw);
}

/* model.py:108-123 */
static dec_t dec_f16(uint32_t bits) {
    bits &= 0xFFFFu;
    int sign = (bits & 0x8000u) ? -1 : 1;
    int exp = (bits >> 10) & 0x1F;
    uint32_t frac = bits & 0x3FFu;
    if (exp == 0x1F) return frac ? special(T_NAN) : special(sign < 0 ? T_NINF : T_PINF);
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 15; }
    else { mant = (1 << 10) | frac; raw = exp - 15; }
    return fin(sign * mant, raw - 10, raw);
}

/* model.py:126-139 */
static dec_t dec_e4m3(uint32_t bits) {
    bits &= 0xFFu;
    int sign = (bits & 0x80u) ? -1 : 1;
    int exp = (bits >> 3) & 0xF;
    uint32_t frac = bits & 0x7u;
    if (exp == 0xF && frac == 0x7) return special(T_NAN);
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 7; }
    else { mant = (1 << 3) | frac; raw = exp - 7; }
    return fin(sign * mant, raw - 3, raw);
}

/* model.py:142-157 */
static dec_t dec_e5m2(uint32_t bits) {
    bits &= 0xFFu;
    int sign = (bits & 0x80u) ? -1 : 1;
    int exp = (bits >> 2) & 0x1F;
    uint32_t frac = bits & 0x3u;
    if (exp == 0x1F) return frac ? special(T_NAN) : special(sign < 0 ? T_NINF : T_PINF);
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 15; }
    else { mant = (1 << 2) | frac; raw = exp - 15; }
    return fin(sign * mant, raw - 2, raw);
}

/* model.py:160-171 */
static dec_t dec_e2m3(uint32_t bits) {
    bits &= 0x3Fu;
    int sign = (bits & 0x20u) ? -1 : 1;
    int exp = (bits >> 3) & 0x3;
    uint32_t frac = bits & 0x7u;
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 1; }
    else { mant = (1 << 3) | frac; raw = exp - 1; }
    return fin(sign * mant, raw - 3, raw);
}

/* model.py:174-185 */
static dec_t dec_e3m2(uint32_t bits) {
    bits &= 0x3Fu;
    int sign = (bits & 0x20u) ? -1 : 1;
    int exp = (bits >> 2) & 0x7;
    uint32_t frac = bits & 0x3u;
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 3; }
    else { mant = (1 << 2) | frac; raw = exp - 3; }
    return fin(sign * mant, raw - 2, raw);
}

/* model.py:188-200 */
static dec_t dec_ue4m3(uint32_t bits) {
    bits &= 0x7Fu;
    int exp = (bits >> 3) & 0xF;
    uint32_t frac = bits & 0x7u;
    if (exp == 0xF && frac == 0x7) return special(T_NAN);
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 7; }
    else { mant = (1 << 3) | frac; raw = exp - 7; }
    return fin(mant, raw - 3, raw);
}

/* model.py:203-208 */
static dec_t dec_ue8m0(uint32_t bits) {
    bits &= 0xFFu;
    if (bits == 0xFF) return special(T_NAN);
    int raw = (int)bits - 127;
    return fin(1, raw, raw);
}

/* model.py:211-222 */
static dec_t dec_e2m1(uint32_t bits) {
    bits &= 0xFu;
    int sign = (bits & 0x8u) ? -1 : 1;
    int exp = (bits >> 1) & 0x3;
    uint32_t frac = bits & 0x1u;
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 1; }
    else { mant = (1 << 1) | frac; raw = exp - 1; }
    return fin(sign * mant, raw - 1, raw);
}

/* model.py:225-239 */
static dec_t dec_f32(uint32_t bits) {
    int sign = (bits & 0x80000000u) ? -1 : 1;
    int exp = (bits & 0x7F800000u) >> 23;
    uint32_t frac = bits & 0x007FFFFFu;
    if (exp == 0xFF) return frac ? special(T_NAN) : special(sign < 0 ? T_NINF : T_PINF);
    int64_t mant; int raw;
    if (exp == 0) { mant = frac; raw = 1 - 127; }
    else { mant = (1 << 23) | frac; raw = exp - 127; }
    return fin(sign * mant, raw - 23, raw);
}

/* model.py:547-564 (_tcgen05_decoder_for_format) plus the per-class decoders */
static dec_t dec_fmt(int fmt, uint32_t bits) {
    switch (fmt) {
    case OF_TF32: return dec_tf32(bits);
    case OF_BF16: return dec_bf16(bits);
    case OF_F16: return dec_f16(bits);
    case OF_E4M3: return dec_e4m3(bits);
    case OF_E5M2: return dec_e5m2(bits);
    case OF_E2M3: return dec_e2m3(bits);
    case OF_E3M2: return dec_e3m2(bits);
    default: return dec_e2m1(bits);
    }
}

/* ---- fixed-point helpers ---- */

static int g_range_error;  /* set when an exactness assumption would fail */

static i128 shl128(i128 v, int s) {
    if (s >= 100) { g_range_error = 1; return 0; }
    return v * ((i128)1 << s);
}
static i128 abs128(i128 v) { return v < 0 ? -v : v; }
static i128 shr_mag(i128 mag, int s) { return s >= 127 ? 0 : (mag >> s); }

/* model.py:242-249 */
static i128 trunc_to_quantum(i128 mant, int value_exp, int quantum_exp) {
    if (mant == 0) return 0;
    int shift = value_exp - quantum_exp;
    if (shift >= 0) return shl128(mant, shift);
    i128 mag = shr_mag(abs128(mant), -shift);
    return mant < 0 ? -mag : mag;
}

/* model.py:263-269: exact sum of (mant, exp) terms at their minimum exponent */
typedef struct { i128 units; int exp; } sum_t;
static sum_t sum_to_common_exp(const i128* mants, const int* exps, int n) {
    sum_t r = {0, 0};
    int have = 0, common = 0;
    for (int i = 0; i < n; i++) {
        if (mants[i] == 0) continue;
        if (!have || exps[i] < common) common = exps[i];
        have = 1;
    }
    if (!have) return r;
    for (int i = 0; i < n; i++) {
        if (mants[i] == 0) continue;
        r.units += shl128(mants[i], exps[i] - common);
    }
    r.exp = common;
    return r;
}

static int bit_length128(i128 mag) {
    int n = 0;
    while (mag > 0) { n++; mag >>= 1; }
    return n;
}

/* model.py:272-307 */
static uint32_t round_to_f32_rz(i128 mant, int value_exp) {
    if (mant == 0) return 0u;
    uint32_t sign_bit = 0;
    if (mant < 0) { sign_bit = 0x80000000u; mant = -mant; }
    int exp = bit_length128(mant) - 1 + value_exp;
    if (exp > 127) return sign_bit | 0x7F800000u;
    if (exp >= -126) {
        int shift = value_exp - exp + 23;
        i128 rm = shift >= 0 ? shl128(mant, shift) : shr_mag(mant, -shift);
        if (rm >= ((i128)1 << 24)) {
            exp += 1;
            rm >>= 1;
            if (exp > 127) return sign_bit | 0x7F800000u;
        }
        return sign_bit | ((uint32_t)(exp + 127) << 23) | ((uint32_t)rm & 0x007FFFFFu);
    }
    int shift = value_exp + 149;
    i128 rm = shift >= 0 ? shl128(mant, shift) : shr_mag(mant, -shift);
    if (rm == 0) return 0u;
    if (rm >= ((i128)1 << 23)) return sign_bit | (1u << 23);
    return sign_bit | (uint32_t)rm;
}

/* model.py:310-321 (mode is always "rne" at the call sites of model.py:628) */
static i128 round_shift_positive(i128 value, int shift, int rne) {
    if (shift <= 0) return shl128(value, -shift);
    i128 q = shr_mag(value, shift);
    if (!rne) return q;
    i128 rem = shift >= 127 ? value : (value & (((i128)1 << shift) - 1));
    i128 twice = rem << 1;
    if (shift >= 126) { /* threshold exceeds every representable remainder */
        return q;
    }
    i128 threshold = (i128)1 << shift;
    if (twice > threshold || (twice == threshold && (q & 1))) return q + 1;
    return q;
}

/* model.py:324-353 */
static uint32_t round_to_f16(i128 mant, int value_exp, int rne) {
    if (mant == 0) return 0u;
    uint32_t sign_bit = 0;
    if (mant < 0) { sign_bit = 0x8000u; mant = -mant; }
    int exp = bit_length128(mant) - 1 + value_exp;
    if (exp > 15) return sign_bit | 0x7C00u;
    if (exp >= -14) {
        int shift = value_exp - exp + 10;
        i128 rm = round_shift_positive(mant, -shift, rne);
        if (rm >= (1 << 11)) {
            exp += 1;
            rm >>= 1;
            if (exp > 15) return sign_bit | 0x7C00u;
        }
        return sign_bit | ((uint32_t)(exp + 15) << 10) | ((uint32_t)rm & 0x03FFu);
    }
    int shift = value_exp + 24;
    i128 rm = round_shift_positive(mant, -shift, rne);
    if (rm == 0) return 0u;
    if (rm >= (1 << 10)) return sign_bit | (1u << 10);
    return sign_bit | (uint32_t)rm;
}

/* ---- model descriptor: the parameters make_model (model.py:1185-1309) picks ---- */
enum { MC_RAW = 1, MC_MIXED = 2, MC_NVFP4 = 3, MC_BLOCK = 4, MC_I8 = 5 };

typedef struct {
    int cls;
    int a_fmt, b_fmt;
    int d_f16;              /* Mixed model with d_type f16 */
    int product_decoder;    /* Mixed model with both formats in the f8f6f4 set */
    int min_window;         /* INT_MIN: None */
    int window_bits;        /* product_window_fraction_bits */
    int scale_ue4m3;        /* block-scaled scale decoder */
    int scale_block, c_merge_group;
    int scale_floor_offset;
    int product_merge_group;  /* 0: None */
    int subnormal_floor;      /* INT_MIN: None */
    int c_merge_bits;
    int use_c_dom, use_pg_c_dom;
    int i8_a_signed, i8_b_signed, saturate;
} omodel_t;

static int is_f8f6f4(int f) { return f >= OF_E4M3 && f <= OF_E2M1; }
static int is_f16in(int f) { return f == OF_BF16 || f == OF_F16; }

static void block_params(omodel_t* m, int a, int b, int block, int cmerge, int wbits, int floor_off,
                         int pmerge, int subfloor, int use_cdom, int use_pgcdom) {
    memset(m, 0, sizeof(*m));
    m->cls = MC_BLOCK; m->a_fmt = a; m->b_fmt = b;
    m->scale_block = block; m->c_merge_group = cmerge; m->window_bits = wbits;
    m->scale_floor_offset = floor_off; m->product_merge_group = pmerge;
    m->subnormal_floor = subfloor; m->c_merge_bits = 35;
    m->use_c_dom = use_cdom; m->use_pg_c_dom = use_pgcdom;
    m->min_window = INT_MIN;
}

/* model.py:1185-1309; b_fmt OF_NONE means "same as A"; scale_vec 0 means None */
static int oracle_make_model(omodel_t* m, int a, int b, int d_type, int saturate,
                             int scaling, int scale_vec, int kind) {
    if (b == OF_NONE) b = a;
    memset(m, 0, sizeof(*m));
    m->min_window = INT_MIN;
    m->subnormal_floor = INT_MIN;
    if (a < OF_TF32 || a > OF_S8 || b < OF_TF32 || b > OF_S8) return ORACLE_ERR_DESCRIPTOR;
    if (d_type < OD_F32 || d_type > OD_S32) return ORACLE_ERR_DESCRIPTOR;
    if (a == OF_U8 || a == OF_S8 || b == OF_U8 || b == OF_S8) {
        if (scaling != OS_NONE || kind != OK_NONE || scale_vec != 0) return ORACLE_ERR_DESCRIPTOR;
        if (!(a == OF_U8 || a == OF_S8) || !(b == OF_U8 || b == OF_S8) || d_type != OD_S32)
            return ORACLE_ERR_DESCRIPTOR;
        m->cls = MC_I8; m->a_fmt = a; m->b_fmt = b;
        m->i8_a_signed = a == OF_S8; m->i8_b_signed = b == OF_S8; m->saturate = saturate != 0;
        return ORACLE_OK;
    }
    if (saturate) return ORACLE_ERR_DESCRIPTOR;
    if (scaling == OS_NONE) {
        if (kind != OK_NONE || scale_vec != 0) return ORACLE_ERR_DESCRIPTOR;
        if (a == OF_TF32 || b == OF_TF32) {
            if (a != OF_TF32 || b != OF_TF32 || d_type != OD_F32) return ORACLE_ERR_DESCRIPTOR;
        } else if (is_f16in(a) || is_f16in(b)) {
            if (a != b || !is_f16in(a)) return ORACLE_ERR_DESCRIPTOR;
            if (d_type == OD_F16 && a != OF_F16) return ORACLE_ERR_DESCRIPTOR;
            if (d_type != OD_F16 && d_type != OD_F32) return ORACLE_ERR_DESCRIPTOR;
        } else if (is_f8f6f4(a) && is_f8f6f4(b)) {
            if (d_type != OD_F16 && d_type != OD_F32) return ORACLE_ERR_DESCRIPTOR;
        } else {
            return ORACLE_ERR_DESCRIPTOR;
        }
        m->a_fmt = a; m->b_fmt = b; m->window_bits = 25;
        if (d_type == OD_F32 && a == b) {   /* FORMAT_MODELS, model.py:1154-1163 */
            m->cls = MC_RAW;
            if (a == OF_TF32 || a == OF_BF16) m->min_window = -133;  /* model.py:462, 476 */
            return ORACLE_OK;
        }
        m->cls = MC_MIXED;                   /* model.py:567-583 */
        m->d_f16 = d_type == OD_F16;
        m->product_decoder = is_f8f6f4(a) && is_f8f6f4(b);
        return ORACLE_OK;
    }
    if (scaling == OS_UE4M3) {
        if (!(kind == OK_NONE || kind == OK_NVFP4 || kind == OK_MXF4NVF4)) return ORACLE_ERR_DESCRIPTOR;
        int sv = scale_vec == 0 ? 4 : scale_vec;
        if (a != OF_E2M1 || b != OF_E2M1 || d_type != OD_F32 || sv != 4) return ORACLE_ERR_DESCRIPTOR;
        memset(m, 0, sizeof(*m));
        m->cls = MC_NVFP4; m->a_fmt = a; m->b_fmt = b;
        m->scale_block = 16; m->c_merge_group = 16;   /* model.py:713 defaults */
        m->min_window = INT_MIN; m->subnormal_floor = INT_MIN;
        return ORACLE_OK;
    }
    if (scaling != OS_UE8M0) return ORACLE_ERR_DESCRIPTOR;
    if (!(kind == OK_NONE || kind == OK_MXF8F6F4 || kind == OK_MXF4 || kind == OK_MXF4NVF4))
        return ORACLE_ERR_DESCRIPTOR;
    if (d_type != OD_F32) return ORACLE_ERR_DESCRIPTOR;
    if (kind == OK_NONE) {
        if (is_f8f6f4(a) && is_f8f6f4(b) && (a != OF_E2M1 || b != OF_E2M1)) kind = OK_MXF8F6F4;
        else return ORACLE_ERR_DESCRIPTOR;
    }
    if (kind == OK_MXF8F6F4) {
        int sv = scale_vec == 0 ? 1 : scale_vec;
        if (sv != 1) return ORACLE_ERR_DESCRIPTOR;
        if (!is_f8f6f4(a) || !is_f8f6f4(b)) return ORACLE_ERR_DESCRIPTOR;
        /* model.py:1008-1075 and 1286-1294: identical parameters for all pairs */
        block_params(m, a, b, 32, 32, 25, 1000, 0, INT_MIN, 0, 0);
        return ORACLE_OK;
    }
    /* kind mxf4 / mxf4nvf4 */
    if (a != OF_E2M1 || b != OF_E2M1) return ORACLE_ERR_DESCRIPTOR;
    int sv = scale_vec == 0 ? 2 : scale_vec;
    if (kind == OK_MXF4) {
        if (sv != 2) return ORACLE_ERR_DESCRIPTOR;
        block_params(m, a, b, 32, 16, 39, 35, 16, -174, 1, 1);   /* model.py:1078-1089 */
        return ORACLE_OK;
    }
    if (sv == 2) { block_params(m, a, b, 32, 16, 39, 35, 16, -174, 1, 1); return ORACLE_OK; } /* :1092 */
    if (sv == 4) { block_params(m, a, b, 16, 16, 39, 35, 16, -174, 1, 1); return ORACLE_OK; } /* :1106 */
    return ORACLE_ERR_DESCRIPTOR;
}

/* ---- one dot product ---- */
typedef struct {
    const uint32_t* a; const uint32_t* b; uint32_t c; int k;
    const uint32_t* scale_a; int nscale_a;   /* NULL: None */
    const uint32_t* scale_b; int nscale_b;
} case_t;

#define CANON_NAN 0x7FFFFFFFu
#define F32_PINF 0x7F800000u
#define F32_NINF 0xFF800000u

/* the sign rules for an infinite product: model.py:393-407 (also :599-613, :879-893) */
static int inf_product(dec_t a, dec_t b, int* out_tag) {
    int a_zero = a.tag == T_FIN && a.mant == 0;
    int b_zero = b.tag == T_FIN && b.mant == 0;
    if (a_zero || b_zero) return 1;  /* NaN */
    int sign = 1;
    if (a.tag == T_NINF) sign = -sign;
    if (b.tag == T_NINF) sign = -sign;
    if (a.tag == T_FIN && a.mant < 0) sign = -sign;
    if (b.tag == T_FIN && b.mant < 0) sign = -sign;
    *out_tag = sign < 0 ? T_NINF : T_PINF;
    return 0;
}

/* raw-window eval, model.py:383-445, and the Mixed override, model.py:644-694 */
static uint32_t eval_raw(const omodel_t* m, const case_t* cs) {
    int mixed_pd = m->cls == MC_MIXED && m->product_decoder;
    uint32_t w_nan = CANON_NAN, w_pinf = F32_PINF, w_ninf = F32_NINF;
    if (mixed_pd && m->d_f16) { w_nan = 0x7FFFu; w_pinf = 0x7C00u; w_ninf = 0xFC00u; }  /* :631-642 */
    int have_pinf = 0, have_ninf = 0;
    int have_raw = 0, max_raw = 0;
    i128* pm = (i128*)malloc(sizeof(i128) * (size_t)(cs->k + 1));
    int* pe = (int*)malloc(sizeof(int) * (size_t)(cs->k + 1));
    int np = 0;
    uint32_t result;
    for (int k = 0; k < cs->k; k++) {
        dec_t a = dec_fmt(m->a_fmt, cs->a[k]);
        dec_t b = dec_fmt(m->b_fmt, cs->b[k]);
        if (a.tag == T_NAN || b.tag == T_NAN) { result = w_nan; goto done; }
        if (a.tag != T_FIN || b.tag != T_FIN) {
            int tag;
            if (inf_product(a, b, &tag)) { result = w_nan; goto done; }
            if (tag == T_PINF) have_pinf = 1; else have_ninf = 1;
            continue;
        }
        i128 mant = (i128)a.mant * b.mant;
        pm[np] = mant; pe[np] = a.ve + b.ve; np++;
        if (mant != 0) {
            int r = a.re + b.re;
            if (!have_raw || r > max_raw) max_raw = r;
            have_raw = 1;
        }
    }
    {
        /* C decode: F32 unless the Mixed model has F16 C/D (model.py:621-624) */
        dec_t c = (m->cls == MC_MIXED && m->d_f16) ? dec_f16(cs->c) : dec_f32(cs->c);
        if (c.tag == T_NAN) { result = w_nan; goto done; }
        if (c.tag == T_PINF) have_pinf = 1;
        if (c.tag == T_NINF) have_ninf = 1;
        if (have_pinf && have_ninf) { result = w_nan; goto done; }   /* _special_sum, model.py:62-69 */
        if (have_pinf) { result = w_pinf; goto done; }
        if (have_ninf) { result = w_ninf; goto done; }
        if (c.tag == T_FIN) {
            pm[np] = c.mant; pe[np] = c.ve; np++;
            if (c.mant != 0) {
                if (!have_raw || c.re > max_raw) max_raw = c.re;
                have_raw = 1;
            }
        }
        if (!have_raw) { result = 0u; goto done; }
        int window = max_raw;
        if (m->min_window != INT_MIN && window < m->min_window) window = m->min_window;  /* :441-442 */
        int q = window - m->window_bits;
        i128 units = 0;
        for (int i = 0; i < np; i++) units += trunc_to_quantum(pm[i], pe[i], q);
        /* output rounding: model.py:380-381 and :626-629 */
        if (m->cls == MC_MIXED && m->d_f16) result = round_to_f16(units, q, 1);
        else result = round_to_f32_rz(units, q);
    }
done:
    free(pm); free(pe);
    return result;
}

/* NVFP4 eval, model.py:721-796 */
static int eval_nvfp4(const omodel_t* m, const case_t* cs, uint32_t* out) {
    int K = cs->k;
    int block_count = (K + m->scale_block - 1) / m->scale_block;
    uint32_t defaults[4096];
    const uint32_t* sa = cs->scale_a; int nsa = cs->nscale_a;
    const uint32_t* sb = cs->scale_b; int nsb = cs->nscale_b;
    if (!sa || !sb) {
        if (block_count > 4096) return ORACLE_ERR_RANGE;
        for (int i = 0; i < block_count; i++) defaults[i] = 0x38;  /* :726-727 */
        if (!sa) { sa = defaults; nsa = block_count; }
        if (!sb) { sb = defaults; nsb = block_count; }
    }
    if (nsa != nsb) return ORACLE_ERR_SCALE_COUNT;
    if ((int64_t)nsa * m->scale_block < K) return ORACLE_ERR_SCALE_COVER;
    i128* pm = (i128*)malloc(sizeof(i128) * (size_t)K);
    int* pe = (int*)malloc(sizeof(int) * (size_t)K);
    int have_prod = 0, max_pr = 0, max_sr = 0;
    uint32_t result;
    for (int k = 0; k < K; k++) {
        dec_t a = dec_e2m1(cs->a[k]);
        dec_t b = dec_e2m1(cs->b[k]);
        int blk = k / m->scale_block;
        dec_t s_a = dec_ue4m3(sa[blk]);
        dec_t s_b = dec_ue4m3(sb[blk]);
        if (s_a.tag == T_NAN || s_b.tag == T_NAN) { result = CANON_NAN; goto done; }
        pm[k] = (i128)a.mant * b.mant * s_a.mant * s_b.mant;
        pe[k] = a.ve + b.ve + s_a.ve + s_b.ve;
        int pr = a.re + b.re + s_a.re + s_b.re;
        int sr = s_a.re + s_b.re;
        if (pm[k] != 0) {
            if (!have_prod || pr > max_pr) max_pr = pr;
            if (!have_prod || sr > max_sr) max_sr = sr;
            have_prod = 1;
        }
    }
    {
        dec_t c = dec_f32(cs->c);
        if (c.tag == T_NAN) { result = CANON_NAN; goto done; }
        if (c.tag == T_PINF) { result = F32_PINF; goto done; }
        if (c.tag == T_NINF) { result = F32_NINF; goto done; }
        if (!have_prod) { result = (cs->c & 0x7FFFFFFFu) == 0 ? 0u : cs->c; goto done; }  /* :768-769 */
        int max_raw = max_pr;
        if (c.mant != 0 && c.re > max_raw) max_raw = c.re;
        if (c.mant != 0 && c.re >= max_pr) {   /* C-dominant: model.py:780-786 */
            int q = c.re - 35;
            i128 units = trunc_to_quantum(c.mant, c.ve, q);
            for (int g = 0; g < K; g += m->c_merge_group) {
                int n = K - g < m->c_merge_group ? K - g : m->c_merge_group;
                sum_t s = sum_to_common_exp(pm + g, pe + g, n);
                units += trunc_to_quantum(s.units, s.exp, q);
            }
            result = round_to_f32_rz(units, q);
            goto done;
        }
        int q = max_raw - 39;                   /* model.py:788 */
        if (max_sr - 35 > q) q = max_sr - 35;
        i128 units = trunc_to_quantum(c.mant, c.ve, q);
        for (int g = 0; g < K; g += 4) {        /* model.py:793-795 */
            int n = K - g < 4 ? K - g : 4;
            sum_t s = sum_to_common_exp(pm + g, pe + g, n);
            units += trunc_to_quantum(s.units, s.exp, q);
        }
        result = round_to_f32_rz(units, q);
    }
done:
    free(pm); free(pe);
    *out = result;
    return ORACLE_OK;
}

/* block-scaled eval, model.py:845-1005 */
static int eval_block(const omodel_t* m, const case_t* cs, uint32_t* out) {
    int K = cs->k;
    int block_count = (K + m->scale_block - 1) / m->scale_block;
    uint32_t defaults[4096];
    const uint32_t* sa = cs->scale_a; int nsa = cs->nscale_a;
    const uint32_t* sb = cs->scale_b; int nsb = cs->nscale_b;
    if (!sa || !sb) {
        if (block_count > 4096) return ORACLE_ERR_RANGE;
        for (int i = 0; i < block_count; i++) defaults[i] = 0x7F;  /* :853-854 */
        if (!sa) { sa = defaults; nsa = block_count; }
        if (!sb) { sb = defaults; nsb = block_count; }
    }
    if (nsa != nsb) return ORACLE_ERR_SCALE_COUNT;
    if ((int64_t)nsa * m->scale_block < K) return ORACLE_ERR_SCALE_COVER;
    i128* pm = (i128*)malloc(sizeof(i128) * (size_t)K);
    int* pe = (int*)malloc(sizeof(int) * (size_t)K);
    int* p_sr = (int*)malloc(sizeof(int) * (size_t)K);   /* INT_MIN: None */
    int* p_pr = (int*)malloc(sizeof(int) * (size_t)K);
    int np = 0;
    int have_pinf = 0, have_ninf = 0, have_prod = 0, max_pr = 0, max_sr = 0;
    uint32_t result;
    for (int k = 0; k < K; k++) {
        dec_t a = dec_fmt(m->a_fmt, cs->a[k]);
        dec_t b = dec_fmt(m->b_fmt, cs->b[k]);
        if (a.tag == T_NAN || b.tag == T_NAN) { result = CANON_NAN; goto done; }
        int blk = k / m->scale_block;
        dec_t s_a = m->scale_ue4m3 ? dec_ue4m3(sa[blk]) : dec_ue8m0(sa[blk]);
        dec_t s_b = m->scale_ue4m3 ? dec_ue4m3(sb[blk]) : dec_ue8m0(sb[blk]);
        if (s_a.tag == T_NAN || s_b.tag == T_NAN) { result = CANON_NAN; goto done; }
        if (a.tag != T_FIN || b.tag != T_FIN) {
            int tag;
            if (inf_product(a, b, &tag)) { result = CANON_NAN; goto done; }
            if (tag == T_PINF) have_pinf = 1; else have_ninf = 1;
            continue;
        }
        i128 mant = (i128)a.mant * b.mant * s_a.mant * s_b.mant;
        int pr = a.re + b.re + s_a.re + s_b.re;
        int sr = s_a.re + s_b.re;
        pm[np] = mant; pe[np] = a.ve + b.ve + s_a.ve + s_b.ve;
        p_sr[np] = mant != 0 ? sr : INT_MIN;
        p_pr[np] = mant != 0 ? pr : INT_MIN;
        np++;
        if (mant != 0) {
            if (!have_prod || pr > max_pr) max_pr = pr;
            if (!have_prod || sr > max_sr) max_sr = sr;
            have_prod = 1;
        }
    }
    {
        dec_t c = dec_f32(cs->c);
        if (c.tag == T_NAN) { result = CANON_NAN; goto done; }
        if (c.tag == T_PINF) have_pinf = 1;
        if (c.tag == T_NINF) have_ninf = 1;
        if (have_pinf && have_ninf) { result = CANON_NAN; goto done; }
        if (have_pinf) { result = F32_PINF; goto done; }
        if (have_ninf) { result = F32_NINF; goto done; }
        if (!have_prod) { result = (cs->c & 0x7FFFFFFFu) == 0 ? 0u : cs->c; goto done; }  /* :926-927 */
        int max_raw = max_pr;
        if (c.mant != 0 && c.re > max_raw) max_raw = c.re;
        /*
         * The C-dominant merge groups and the product groups below index the
         * product list by position.  The reference appends to merge_groups by
         * k (model.py:904) but slices `products` by position (model.py:952);
         * both agree because an infinite operand never reaches this point
         * (it either returned NaN or a signed infinity above).
         */
        if (m->use_c_dom && c.mant != 0 && c.re >= max_pr) {   /* model.py:934-940 */
            int q = c.re - m->c_merge_bits;
            i128 units = trunc_to_quantum(c.mant, c.ve, q);
            for (int g = 0; g < np; g += m->c_merge_group) {
                int n = np - g < m->c_merge_group ? np - g : m->c_merge_group;
                sum_t s = sum_to_common_exp(pm + g, pe + g, n);
                units += trunc_to_quantum(s.units, s.exp, q);
            }
            result = round_to_f32_rz(units, q);
            goto done;
        }
        int q = max_raw - m->window_bits;                       /* model.py:942-945 */
        if (max_sr - m->scale_floor_offset > q) q = max_sr - m->scale_floor_offset;
        i128 c_units = trunc_to_quantum(c.mant, c.ve, q);
        i128 units = c_units;
        if (m->product_merge_group == 0) {                      /* model.py:947-948 */
            for (int i = 0; i < np; i++) units += trunc_to_quantum(pm[i], pe[i], q);
            result = round_to_f32_rz(units, q);
            goto done;
        }
        int G = m->product_merge_group;
        int ngroups = (np + G - 1) / G;
        i128* bu = (i128*)malloc(sizeof(i128) * (size_t)(ngroups + 1));
        int* gsr = (int*)malloc(sizeof(int) * (size_t)(ngroups + 1));
        for (int gi = 0; gi < ngroups; gi++) {                   /* model.py:951-983 */
            int g = gi * G;
            int n = np - g < G ? np - g : G;
            sum_t s = sum_to_common_exp(pm + g, pe + g, n);
            int g_sr = INT_MIN, g_pr = INT_MIN;
            for (int i = g; i < g + n; i++) {
                if (p_sr[i] != INT_MIN && (g_sr == INT_MIN || p_sr[i] > g_sr)) g_sr = p_sr[i];
                if (p_pr[i] != INT_MIN && (g_pr == INT_MIN || p_pr[i] > g_pr)) g_pr = p_pr[i];
            }
            int bq = q;
            if (m->use_pg_c_dom && c.mant != 0 && g_pr != INT_MIN && c.re >= g_pr) {
                int cq = c.re - m->c_merge_bits;
                if (cq > bq) bq = cq;
            }
            i128 b_units = trunc_to_quantum(s.units, s.exp, bq);
            b_units = shl128(b_units, bq - q);
            bu[gi] = b_units; gsr[gi] = g_sr;
            units += b_units;
        }
        result = round_to_f32_rz(units, q);
        if (m->subnormal_floor != INT_MIN) {                      /* model.py:986-1003 */
            uint32_t mag = result & 0x7FFFFFFFu;
            if (mag > 0 && mag < (1u << 23)) {
                /* threshold_units = 2**(floor - q) or 1; compared through bit lengths so
                   that thresholds beyond the __int128 range stay exact */
                int thr_bits = q < m->subnormal_floor ? m->subnormal_floor - q : 0;
                i128 filtered = c_units;
                for (int gi = 0; gi < ngroups; gi++) {
                    int below = bit_length128(abs128(bu[gi])) <= thr_bits;   /* |bu| < 2**thr_bits */
                    if (gsr[gi] != INT_MIN && gsr[gi] < max_sr && below) continue;
                    filtered += bu[gi];
                }
                result = round_to_f32_rz(filtered, q);
            }
        }
        free(bu); free(gsr);
    }
done:
    free(pm); free(pe); free(p_sr); free(p_pr);
    *out = result;
    return ORACLE_OK;
}

/* model.py:1120-1152 */
static uint32_t eval_i8(const omodel_t* m, const case_t* cs) {
    int64_t total = (int64_t)(int32_t)cs->c;
    for (int k = 0; k < cs->k; k++) {
        int64_t a = cs->a[k] & 0xFF, b = cs->b[k] & 0xFF;
        if (m->i8_a_signed && (a & 0x80)) a -= 0x100;
        if (m->i8_b_signed && (b & 0x80)) b -= 0x100;
        total += a * b;
    }
    if (m->saturate) {
        if (total < -(int64_t)0x80000000LL) total = -(int64_t)0x80000000LL;
        if (total > 0x7FFFFFFFLL) total = 0x7FFFFFFFLL;
    }
    return (uint32_t)(total & 0xFFFFFFFFLL);
}

/* ScalarModel.eval dispatch */
static int oracle_eval(const omodel_t* m, const case_t* cs, uint32_t* out) {
    if (cs->k <= 0) return ORACLE_ERR_EMPTY;                         /* model.py:35-36 */
    if ((cs->scale_a == NULL) != (cs->scale_b == NULL)) return ORACLE_ERR_SCALE_PAIR;  /* :40-41 */
    for (int i = 0; cs->scale_a && i < cs->nscale_a; i++)                           /* :42-44 */
        if (cs->scale_a[i] > 0xFFu) return ORACLE_ERR_SCALE_VALUE;
    for (int i = 0; cs->scale_b && i < cs->nscale_b; i++)
        if (cs->scale_b[i] > 0xFFu) return ORACLE_ERR_SCALE_VALUE;
    switch (m->cls) {
    case MC_RAW:
    case MC_MIXED: *out = eval_raw(m, cs); return ORACLE_OK;
    case MC_NVFP4: return eval_nvfp4(m, cs, out);
    case MC_BLOCK: return eval_block(m, cs, out);
    default: *out = eval_i8(m, cs); return ORACLE_OK;
    }
}

/*
 * sparse_active_indices, simulator.py:26-77.  Fills `active` (a bitmap over
 * logical K) and returns the status.  `meta_is_int` mirrors an int argument
 * (a single word repeated to cover K, simulator.py:58-59).
 */
static int active_indices(int a_fmt, int k, const uint32_t* words, int nwords, int meta_is_int,
                          int kind, int nvfp4, unsigned char* active) {
    if (!(kind == OK_NONE || kind == OK_MXF8F6F4 || kind == OK_MXF4 || kind == OK_MXF4NVF4 || kind == OK_NVFP4))
        return ORACLE_ERR_KIND;
    int pairwise = nvfp4 || kind == OK_MXF4 || kind == OK_MXF4NVF4 || kind == OK_NVFP4;
    if (nwords <= 0) return ORACLE_ERR_META_WORDS;
    int chunk_size, chunks, tf32 = a_fmt == OF_TF32;
    if (tf32) { chunk_size = 2; chunks = (k + 1) / 2; }
    else { chunk_size = pairwise ? 8 : 4; chunks = (k + chunk_size - 1) / chunk_size; }
    (void)chunk_size;
    int64_t total_words = meta_is_int ? (int64_t)((chunks + 7) / 8) : nwords;
    if (total_words * 8 < chunks) return ORACLE_ERR_META_WORDS;
    memset(active, 0, (size_t)k);
    for (int chunk = 0; chunk < chunks; chunk++) {
        uint32_t word = meta_is_int ? words[0] : words[chunk / 8];
        uint32_t sel = (word >> ((chunk & 7) * 4)) & 0xFu;
        if (tf32) {
            if (!(sel == 0x4 || sel == 0xE)) return ORACLE_ERR_SELECTOR;
            int idx = chunk * 2 + (sel == 0xE);
            if (idx < k) active[idx] = 1;
            continue;
        }
        if (!(sel == 0x4 || sel == 0x8 || sel == 0xC || sel == 0x9 || sel == 0xD || sel == 0x6 || sel == 0xE))
            return ORACLE_ERR_SELECTOR;
        int first = sel & 3, second = (sel >> 2) & 3;
        int idx[4]; int n;
        if (pairwise) {
            idx[0] = chunk * 8 + first * 2; idx[1] = idx[0] + 1;
            idx[2] = chunk * 8 + second * 2; idx[3] = idx[2] + 1; n = 4;
        } else {
            idx[0] = chunk * 4 + first; idx[1] = chunk * 4 + second; n = 2;
        }
        for (int i = 0; i < n; i++) if (idx[i] < k) active[idx[i]] = 1;
    }
    return ORACLE_OK;
}

/* ---- public batch entry: mma_dot (simulator.py:80-140) over N cases ---- */
typedef struct {
    int a_fmt, b_fmt, d_type, saturate, scaling, scale_vec, kind;
} oracle_desc;

static int mma_dot_one(const omodel_t* model, const oracle_desc* d, int k,
                       const uint32_t* a, const uint32_t* b, uint32_t c,
                       const uint32_t* sa, int nsa, const uint32_t* sb, int nsb,
                       const uint32_t* meta, int nmeta, int meta_is_int,
                       uint32_t* out) {
    case_t cs;
    memset(&cs, 0, sizeof(cs));
    cs.c = c;
    cs.scale_a = sa; cs.nscale_a = nsa; cs.scale_b = sb; cs.nscale_b = nsb;
    if (meta == NULL) {
        cs.a = a; cs.b = b; cs.k = k;
        return oracle_eval(model, &cs, out);
    }
    unsigned char stack_active[512];
    uint32_t stack_a[512], stack_b[512];
    unsigned char* active = k <= 512 ? stack_active : (unsigned char*)malloc((size_t)k);
    uint32_t* wa = k <= 512 ? stack_a : (uint32_t*)malloc(sizeof(uint32_t) * (size_t)k);
    uint32_t* wb = k <= 512 ? stack_b : (uint32_t*)malloc(sizeof(uint32_t) * (size_t)k);
    int kind_for_meta = d->scaling == OS_UE4M3 ? OK_NVFP4 : d->kind;   /* simulator.py:113 */
    int st = active_indices(d->a_fmt, k, meta, nmeta, meta_is_int, kind_for_meta, 0, active);
    if (st == ORACLE_OK) {
        int n = 0;
        if (d->scaling == OS_NONE) {          /* simulator.py:115-117: mask at logical K */
            for (int i = 0; i < k; i++) { wa[i] = active[i] ? a[i] : 0; wb[i] = active[i] ? b[i] : 0; }
            n = k;
        } else {                              /* simulator.py:118-121: compress to physical K */
            for (int i = 0; i < k; i++) if (active[i]) { wa[n] = a[i]; wb[n] = b[i]; n++; }
        }
        cs.a = wa; cs.b = wb; cs.k = n;
        st = oracle_eval(model, &cs, out);
    }
    if (k > 512) { free(active); free(wa); free(wb); }
    return st;
}

/*
 * Evaluate n independent mma_dot calls.  a, b: [n][k] raw words; c: [n];
 * scale_a/scale_b: [n][nscale_*] or NULL; meta: [n][nmeta] or NULL.
 * d receives the result words; status (may be NULL) the per-case status.
 * Returns the descriptor status (make_model) or the count of failing cases.
 */
int oracle_mma_dot_batch(const oracle_desc* desc, int64_t n, int k,
                         const uint32_t* a, const uint32_t* b, const uint32_t* c,
                         const uint32_t* scale_a, int nscale_a,
                         const uint32_t* scale_b, int nscale_b,
                         const uint32_t* meta, int nmeta, int meta_is_int,
                         uint32_t* d, int32_t* status, int threads) {
    omodel_t model;
    /* simulator.py:109-114 runs sparse_active_indices (and its kind check) before make_model */
    if (meta != NULL) {
        int kind_for_meta = desc->scaling == OS_UE4M3 ? OK_NVFP4 : desc->kind;
        if (!(kind_for_meta == OK_NONE || kind_for_meta == OK_MXF8F6F4 || kind_for_meta == OK_MXF4 ||
              kind_for_meta == OK_MXF4NVF4 || kind_for_meta == OK_NVFP4))
            return ORACLE_ERR_KIND;
    }
    int st = oracle_make_model(&model, desc->a_fmt, desc->b_fmt, desc->d_type, desc->saturate,
                               desc->scaling, desc->scale_vec, desc->kind);
    if (st != ORACLE_OK) return st;
    g_range_error = 0;
    int64_t failures = 0;
    if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 256) reduction(+ : failures)
    for (int64_t i = 0; i < n; i++) {
        uint32_t out = 0;
        int s = mma_dot_one(&model, desc, k, a + i * k, b + i * k, c[i],
                            scale_a ? scale_a + i * nscale_a : NULL, nscale_a,
                            scale_b ? scale_b + i * nscale_b : NULL, nscale_b,
                            meta ? meta + i * nmeta : NULL, nmeta, meta_is_int, &out);
        d[i] = s == ORACLE_OK ? out : 0u;
        if (status) status[i] = s;
        if (s != ORACLE_OK) failures++;
    }
    if (g_range_error) return ORACLE_ERR_RANGE;
    return (int)(failures > 0x7FFFFFFF ? 0x7FFFFFFF : failures);
}

/* make_model's legality check alone (model.py:1185-1309) */
int oracle_check_descriptor(const oracle_desc* desc) {
    omodel_t model;
    return oracle_make_model(&model, desc->a_fmt, desc->b_fmt, desc->d_type, desc->saturate,
                             desc->scaling, desc->scale_vec, desc->kind);
}

/* sparse_active_indices (simulator.py:26-77): writes a 0/1 map of length k */
int oracle_sparse_active(int a_fmt, int k, const uint32_t* words, int nwords, int meta_is_int,
                         int kind, int nvfp4, unsigned char* active) {
    return active_indices(a_fmt, k, words, nwords, meta_is_int, kind, nvfp4, active);
}
