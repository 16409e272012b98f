/*
 * oracle/nvfp4_ref.c -- CPU restatement of the NVFP4 quantiser.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path (demon_b200/) links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference leg of bench.py use it, as the checker.
 *
 * The reference (daydreamlive/DEMON) has no NVFP4 code.  Its only low-precision
 * linear recipe is FP8 E4M3 with a per-output-channel scale
 * (acestep/engine/trt/fp8_onnx.py:115-149: scale = max(absmax, 1e-12) / 448,
 * torch.float8_e4m3fn round-to-nearest-even cast).  This file restates the
 * public NVFP4 format with the reference's conventions pinned wherever the
 * reference has one:
 *
 *   - absmax floor 1e-12                      (fp8_onnx.py:67 _ABSMAX_FLOOR)
 *   - E4M3 max 448, RNE cast, clamp BEFORE the cast
 *                                             (fp8_onnx.py:61, :144-146;
 *                                              lora_refit.py:598-601 clamps
 *                                              before the cast the same way)
 *   - global scale g = max(amax, 1e-12) / (6 * 448)
 *   - 16-element blocks along K, E4M3 block scale
 *       s_b  = e4m3_rne(min(amax_b / (6 g), 448))
 *       code = e2m1_rne(x * (1 / (f32(s_b) * g)))   (saturating at 6)
 *   - E2M1 magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, ties to the even code,
 *     a value that rounds to zero is always code 0 (no negative zero),
 *     NaN inputs give code 0.
 *   - codes packed two per byte, element 2j in the low nibble.
 *
 * The E4M3 part is pinned against torch's float8_e4m3fn cast (the conversion
 * the reference uses) by tests/test_oracle_nvfp4.py.  The E2M1 part has no
 * reference implementation to pin against ("parity unpinned" for that half);
 * it is checked against a second, independent numpy restatement and a
 * known-answer table instead.
 *
 * Every arithmetic step is a single IEEE-754 binary32 operation with
 * round-to-nearest-even, in the order written, so that the CUDA kernel
 * (demon_b200/csrc/nvfp4_quant.cu) can reproduce it bit for bit.  Build with
 * -ffp-contract=off and without -ffast-math.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define NVFP4_BLOCK 16
#define E4M3_MAX 448.0f
#define ABSMAX_FLOOR 1e-12f
#define GS_DENOM 2688.0f /* 6 * 448 */

enum { GS_STATIC = 0, GS_DYNAMIC = 1, GS_PER_ROW = 2 };

static float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round-to-nearest-even float -> E4M3FN (bias 7, 3 mantissa bits, max 448,
 * subnormals k * 2^-9).  Values at or above the 448/480 midpoint saturate to
 * 448 (satfinite); callers clamp to 448 first anyway. */
uint8_t demon_oracle_e4m3_encode(float x) {
    uint8_t sign = signbit(x) ? 0x80 : 0x00;
    float a = fabsf(x);
    if (isnan(a)) return 0x7f;
    if (a >= 464.0f) return (uint8_t)(sign | 0x7e);
    if (a < 0.015625f) {                      /* below 2^-6: subnormal grid */
        float k = rintf(a * 512.0f);          /* exact scaling, RNE */
        return (uint8_t)(sign | (uint8_t)k);  /* k == 8 is the min normal 0x08 */
    }
    int e;
    float m = frexpf(a, &e);                  /* a = m * 2^e, m in [0.5, 1) */
    float q = rintf(m * 16.0f);               /* 3 mantissa bits + hidden, RNE */
    if (q >= 16.0f) { q = 8.0f; e += 1; }
    int exp_field = e - 1 + 7;
    int mant = (int)q - 8;
    return (uint8_t)(sign | (exp_field << 3) | mant);
}

float demon_oracle_e4m3_decode(uint8_t b) {
    int s = (b >> 7) & 1, e = (b >> 3) & 0xf, m = b & 7;
    float v;
    if (e == 0xf && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);
    else v = ldexpf((float)(8 + m), e - 10);
    return s ? -v : v;
}

uint8_t demon_oracle_e2m1_encode(float v) {
    float a = fabsf(v);
    uint8_t mag;
    if (!(a > 0.25f)) mag = 0;
    else if (a < 0.75f) mag = 1;
    else if (a <= 1.25f) mag = 2;
    else if (a < 1.75f) mag = 3;
    else if (a <= 2.5f) mag = 4;
    else if (a < 3.5f) mag = 5;
    else if (a <= 5.0f) mag = 6;
    else mag = 7;
    return (mag != 0 && v < 0.0f) ? (uint8_t)(mag | 8) : mag;
}

float demon_oracle_e2m1_decode(uint8_t c) {
    static const float lut[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    float v = lut[c & 7];
    return (c & 8) ? -v : v;
}

float demon_oracle_global_scale(float amax) {
    float a = amax > ABSMAX_FLOOR ? amax : ABSMAX_FLOOR;
    return a / GS_DENOM;
}

/* Byte offset of the block scale of (row m, 16-element block kb) in the
 * tcgen05 scale-factor layout: 128-row x 64-element chunks of 512 bytes,
 * inside a chunk row r sits at (r%32)*16 + (r/32)*4 and block kb%4 at +kb%4. */
int64_t demon_oracle_sf_offset(int64_t m, int64_t kb, int64_t K) {
    int64_t chunk = (m / 128) * (K / 64) + kb / 4;
    int64_t r = m % 128;
    return chunk * 512 + (r % 32) * 16 + (r / 32) * 4 + (kb % 4);
}

int64_t demon_oracle_sf_bytes(int64_t rows, int64_t K) {
    return ((rows + 127) / 128) * 128 * (K / NVFP4_BLOCK);
}

static void quantize_row(const uint16_t* xr, int64_t K, float g, uint8_t* code_row,
                         uint8_t* sf_row_lin, int64_t m, uint8_t* sf_swz) {
    float denom = 6.0f * g;
    for (int64_t kb = 0; kb < K / NVFP4_BLOCK; ++kb) {
        float xs[NVFP4_BLOCK];
        float amax = 0.0f;
        for (int i = 0; i < NVFP4_BLOCK; ++i) {
            xs[i] = bf16_to_f32(xr[kb * NVFP4_BLOCK + i]);
            float a = fabsf(xs[i]);
            if (a > amax) amax = a;           /* NaN never wins (same as fmaxf) */
        }
        float s = amax / denom;
        if (!(s <= E4M3_MAX)) s = E4M3_MAX;   /* clamp before the cast */
        uint8_t sb = demon_oracle_e4m3_encode(s);
        float sbf = demon_oracle_e4m3_decode(sb);
        if (sf_row_lin) sf_row_lin[kb] = sb;
        if (sf_swz) sf_swz[demon_oracle_sf_offset(m, kb, K)] = sb;
        uint8_t codes[NVFP4_BLOCK];
        if (sbf == 0.0f) {
            memset(codes, 0, sizeof codes);
        } else {
            float scale = sbf * g;
            float rs = 1.0f / scale;
            for (int i = 0; i < NVFP4_BLOCK; ++i) codes[i] = demon_oracle_e2m1_encode(xs[i] * rs);
        }
        for (int i = 0; i < NVFP4_BLOCK / 2; ++i)
            code_row[kb * (NVFP4_BLOCK / 2) + i] = (uint8_t)(codes[2 * i] | (codes[2 * i + 1] << 4));
    }
}

static float row_amax(const uint16_t* xr, int64_t K) {
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
        float a = fabsf(bf16_to_f32(xr[k]));
        if (a > amax) amax = a;
    }
    return amax;
}

/* x: bf16 bits [M, ldx]; codes [M, K/2]; sf_swz: tcgen05 layout
 * (demon_oracle_sf_bytes(M, K) bytes, pad rows written as 0) or NULL;
 * sf_lin: row-major [M, K/16] or NULL.  gs: static -> gs[0] read;
 * dynamic -> gs[0] written; per-row -> gs[0..M) written. */
int demon_oracle_quantize(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, int gs_mode,
                          float* gs, uint8_t* codes, uint8_t* sf_swz, uint8_t* sf_lin) {
    if (K % 64 != 0 || M < 0 || ldx < K) return 1;
    if (sf_swz) memset(sf_swz, 0, (size_t)demon_oracle_sf_bytes(M, K));
    float g = 0.0f;
    if (gs_mode == GS_STATIC) {
        g = gs[0];
    } else if (gs_mode == GS_DYNAMIC) {
        float amax = 0.0f;
        for (int64_t m = 0; m < M; ++m) {
            float a = row_amax(x + m * ldx, K);
            if (a > amax) amax = a;
        }
        g = demon_oracle_global_scale(amax);
        gs[0] = g;
    } else if (gs_mode != GS_PER_ROW) {
        return 1;
    }
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * ldx;
        float gm = g;
        if (gs_mode == GS_PER_ROW) {
            gm = demon_oracle_global_scale(row_amax(xr, K));
            gs[m] = gm;
        }
        quantize_row(xr, K, gm, codes + m * (K / 2), sf_lin ? sf_lin + m * (K / 16) : NULL, m, sf_swz);
    }
    return 0;
}

/* Dequantise codes + row-major block scales to fp32 [M, K]:
 * x_hat = e2m1(code) * f32(s_b) * g_row. */
void demon_oracle_dequant(const uint8_t* codes, const uint8_t* sf_lin, const float* gs,
                          int gs_per_row, int64_t M, int64_t K, float* out) {
    for (int64_t m = 0; m < M; ++m) {
        float g = gs[gs_per_row ? m : 0];
        for (int64_t k = 0; k < K; ++k) {
            uint8_t byte = codes[m * (K / 2) + k / 2];
            uint8_t c = (k & 1) ? (byte >> 4) : (byte & 0xf);
            float sb = demon_oracle_e4m3_decode(sf_lin[m * (K / 16) + k / 16]);
            out[m * K + k] = demon_oracle_e2m1_decode(c) * sb * g;
        }
    }
}
