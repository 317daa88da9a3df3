/*
 * vbq_oracle.c -- CPU restatement of VibeBlade's GGUF k-quant dequantize-and-multiply path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA product in
 * vibeblade_b200/csrc; nothing in the product links or calls it.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Parity is pinned: tests/test_oracle.py checks every function here bit-exactly
 * against the reference's own C++ compiled from its sources (oracle/_ref, built by
 * oracle/build.py) and against the committed golden vectors in tests/golden/.
 *
 * Each function restates the reference algorithm it cites (path within the
 * kevin046/VibeBlade project).  Compile with -ffp-contract=off so the C compiler
 * never fuses a multiply and an add that the reference evaluates separately.
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <math.h>

/* ggml type ids: cpp/include/ggml_types.h:11-27 */
enum {
    VBO_F32 = 0, VBO_F16 = 1, VBO_Q4_0 = 2, VBO_Q4_1 = 3, VBO_Q5_0 = 6, VBO_Q5_1 = 7,
    VBO_Q8_0 = 8, VBO_Q2_K = 10, VBO_Q3_K = 11, VBO_Q4_K = 12, VBO_Q5_K = 13, VBO_Q6_K = 14,
    VBO_Q8_K = 15, VBO_BF16 = 30
};

/* Block geometry: cpp/include/ggml_types.h:31-71 (values per block 1 / 32 / 256; bytes per
 * block as the size table lists them, Q8_0 the 34-byte GGUF block, Q8_K 292). */
int64_t vbo_block_values(int32_t type) {
    switch (type) {
        case VBO_F32: case VBO_F16: case VBO_BF16: return 1;
        case VBO_Q4_0: case VBO_Q4_1: case VBO_Q5_0: case VBO_Q5_1: case VBO_Q8_0: return 32;
        case VBO_Q2_K: case VBO_Q3_K: case VBO_Q4_K: case VBO_Q5_K: case VBO_Q6_K: case VBO_Q8_K:
            return 256;
        default: return -1;
    }
}

int64_t vbo_block_bytes(int32_t type) {
    switch (type) {
        case VBO_F32: return 4;
        case VBO_F16: case VBO_BF16: return 2;
        case VBO_Q4_0: return 18;
        case VBO_Q4_1: return 20;
        case VBO_Q5_0: return 22;
        case VBO_Q5_1: return 24;
        case VBO_Q8_0: return 34;
        case VBO_Q2_K: return 84;
        case VBO_Q3_K: return 110;
        case VBO_Q4_K: return 144;
        case VBO_Q5_K: return 176;
        case VBO_Q6_K: return 210;
        case VBO_Q8_K: return 292;
        default: return -1;
    }
}

/* Row stride used by gemv_dequant: (N / block_values) * block_bytes, truncating
 * (cpp/src/dequant.cpp:749-763). */
int64_t vbo_row_bytes(int32_t type, int64_t n) {
    int64_t bv = vbo_block_values(type), bb = vbo_block_bytes(type);
    if (bv <= 0) return -1;
    return (n / bv) * bb;
}

/* fp16 -> fp32 as the reference's f16_to_f32 computes it (cpp/src/fp16_compat.cpp:13-35),
 * written as bit arithmetic on the fields.  Normal numbers, zeros, inf and NaN payloads
 * convert exactly.  Subnormals do not: the reference normalises the mantissa starting
 * from exponent 1 and then adds one more to the bias (`exp + 127 - 15 + 1`), so every
 * subnormal input comes out twice its IEEE value.  The k-quant dequantizers that call it
 * (Q4_K d/dmin, Q6_K d) inherit that factor, and parity is defined against them. */
float vbo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0x1fu) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        /* IEEE value m * 2^-24 has biased fp32 exponent 113 - shift; the reference
         * produces 114 - shift. */
        int shift = 0;
        while ((m & 0x400u) == 0) { m <<= 1; ++shift; }
        bits = sign | ((uint32_t)(114 - shift) << 23) | ((m & 0x3ffu) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Exact IEEE fp16 -> fp32 (subnormals included), the conversion the reference's CUDA
 * kernels (__half2float, cpp/src/cuda_kernels.cu:731) and numpy loader
 * (np.float16, vibeblade/loader.py:131) use for the Q8_0 scale. */
float vbo_f16_to_f32_ieee(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0x1fu) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        int shift = 0;
        while ((m & 0x400u) == 0) { m <<= 1; ++shift; }
        bits = sign | ((uint32_t)(113 - shift) << 23) | ((m & 0x3ffu) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* 6-bit scale/min unpacking of a Q4_K super-block (cpp/src/dequant.cpp:258-266). */
static void q4k_scale_min(int j, const uint8_t* s, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Q4_K: 144-byte block = d(f16) @0, dmin(f16) @2, scales[12] @4, qs[128] @16.
 * Four 64-value groups g: byte qs[32g+l] holds value 64g+l (low nibble, scale pair 2g)
 * and 64g+32+l (high nibble, pair 2g+1); out = (d*sc)*q - dmin*m
 * (cpp/src/dequant.cpp:268-301). */
void vbo_dequantize_row_q4_K(const uint8_t* row, float* out, int64_t n) {
    int64_t nb = (n + 255) / 256;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * 144;
        float d = vbo_f16_to_f32(rd16(blk));
        float dmin = vbo_f16_to_f32(rd16(blk + 2));
        const uint8_t* sc = blk + 4;
        const uint8_t* qs = blk + 16;
        for (int g = 0; g < 4; ++g) {
            int s0, m0, s1, m1;
            q4k_scale_min(2 * g, sc, &s0, &m0);
            q4k_scale_min(2 * g + 1, sc, &s1, &m1);
            float dl = d * (float)s0, ml = dmin * (float)m0;
            float dh = d * (float)s1, mh = dmin * (float)m1;
            for (int l = 0; l < 32; ++l) {
                int64_t i_lo = b * 256 + 64 * g + l;
                int64_t i_hi = i_lo + 32;
                float prod_lo = dl * (float)(qs[32 * g + l] & 0x0f);
                float prod_hi = dh * (float)(qs[32 * g + l] >> 4);
                if (i_lo < n) out[i_lo] = prod_lo - ml;
                if (i_hi < n) out[i_hi] = prod_hi - mh;
            }
        }
    }
}

/* Q6_K (reference layout, not llama.cpp's): 210-byte block = ql[128] @0, qh[64] @128,
 * int8 scales[16] @192, d(f16) @208.  Value i: low 4 bits = nibble (i&1) of ql[i>>1],
 * high 2 bits = field (i&3) of qh[i>>2] (LSB first), q = that - 32,
 * out = (d*scale[i>>4])*q (cpp/src/dequant.cpp:359-402; the 4-way ql index branch at
 * :379-394 reduces to i>>1). */
void vbo_dequantize_row_q6_K(const uint8_t* row, float* out, int64_t n) {
    int64_t nb = (n + 255) / 256;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * 210;
        float d = vbo_f16_to_f32(rd16(blk + 208));
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        int64_t rem = n - b * 256;
        if (rem > 256) rem = 256;
        for (int64_t i = 0; i < rem; ++i) {
            int lo = (ql[i >> 1] >> (4 * (i & 1))) & 0x0f;
            int hi = (qh[i >> 2] >> (2 * (i & 3))) & 0x03;
            int q = (lo | (hi << 4)) - 32;
            float ds = d * (float)sc[i >> 4];
            out[b * 256 + i] = ds * (float)q;
        }
    }
}

/* Q8_0 with the GGUF block: fp16 d @0, int8 qs[32] @2, 34-byte stride; out = qs[i]*d.
 * Follows the reference's CUDA kernel (cpp/src/cuda_kernels.cu:718-735) and Python
 * loader (vibeblade/loader.py:129-133).  The C++ CPU dequantize_row_q8_0
 * (cpp/src/dequant.cpp:99-112) reads a 4-byte float scale instead; that variant is
 * restated below as vbo_dequantize_row_q8_0_f32scale to document the defect. */
void vbo_dequantize_row_q8_0(const uint8_t* row, float* out, int64_t n) {
    int64_t nb = (n + 31) / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * 34;
        float d = vbo_f16_to_f32_ieee(rd16(blk));
        const int8_t* qs = (const int8_t*)(blk + 2);
        int64_t rem = n - b * 32;
        if (rem > 32) rem = 32;
        for (int64_t i = 0; i < rem; ++i) out[b * 32 + i] = (float)qs[i] * d;
    }
}

/* The C++ CPU reading of a Q8_0 block (cpp/src/dequant.cpp:99-112): float32 d from
 * bytes 0-3, quants from byte 4 on, stride 34 (overlaps the next block by 2 bytes). */
void vbo_dequantize_row_q8_0_f32scale(const uint8_t* row, float* out, int64_t n) {
    int64_t nb = (n + 31) / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * 34;
        float d;
        memcpy(&d, blk, 4);
        const int8_t* qs = (const int8_t*)(blk + 4);
        int64_t rem = n - b * 32;
        if (rem > 32) rem = 32;
        for (int64_t i = 0; i < rem; ++i) out[b * 32 + i] = (float)qs[i] * d;
    }
}

/* Unquantized rows (cpp/src/dequant.cpp:407-411): F32 copied, F16 through the
 * reference's own conversion (so subnormals double, fp16_compat.cpp:13-35), BF16 as the
 * top half of an fp32 (bf16_to_f32, cpp/include/ggml_types.h:175-180). */
static void vbo_row_f32(const uint8_t* row, float* out, int64_t n) { memcpy(out, row, (size_t)n * 4); }
static void vbo_row_f16(const uint8_t* row, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = vbo_f16_to_f32(rd16(row + 2 * i));
}
static void vbo_row_bf16(const uint8_t* row, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const uint32_t bits = (uint32_t)rd16(row + 2 * i) << 16;
        memcpy(out + i, &bits, 4);
    }
}

/* ---- the other block types of the reference's dispatcher (cpp/src/dequant.cpp:407-425) ----
 * Each restates the reference's reading of its block, which is not always llama.cpp's:
 * the index formulas below are the reference's loops solved for one value index.  fp16
 * fields go through the reference's f16_to_f32 (subnormals doubled); every product and
 * sum the reference writes as separate operations is rounded separately. */

static int64_t rem_of(int64_t n, int64_t b, int64_t bv) {
    int64_t r = n - b * bv;
    return r > bv ? bv : r;
}

/* Q4_0, 18 B: d(f16) @0, qs[16] @2; value i = nibble (i&1) of qs[i>>1]; out = (q-8)*d
 * (cpp/src/dequant.cpp:23-35). */
void vbo_dequantize_row_q4_0(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 32 < n; ++b) {
        const uint8_t* blk = row + b * 18;
        float d = vbo_f16_to_f32(rd16(blk));
        for (int64_t i = 0; i < rem_of(n, b, 32); ++i) {
            int q = (blk[2 + (i >> 1)] >> (4 * (i & 1))) & 15;
            out[b * 32 + i] = (float)(q - 8) * d;
        }
    }
}

/* Q4_1, 20 B: d @0, m @2 (f16), qs[16] @4; out = d*q + m (cpp/src/dequant.cpp:40-53). */
void vbo_dequantize_row_q4_1(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 32 < n; ++b) {
        const uint8_t* blk = row + b * 20;
        float d = vbo_f16_to_f32(rd16(blk)), m = vbo_f16_to_f32(rd16(blk + 2));
        for (int64_t i = 0; i < rem_of(n, b, 32); ++i) {
            int q = (blk[4 + (i >> 1)] >> (4 * (i & 1))) & 15;
            float p = d * (float)q;
            out[b * 32 + i] = p + m;
        }
    }
}

/* Q5_0, 22 B: d @0, qh[4] @2 (bit i = fifth bit of value i), qs[16] @6;
 * out = (q-16)*d (cpp/src/dequant.cpp:58-73). */
void vbo_dequantize_row_q5_0(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 32 < n; ++b) {
        const uint8_t* blk = row + b * 22;
        float d = vbo_f16_to_f32(rd16(blk));
        for (int64_t i = 0; i < rem_of(n, b, 32); ++i) {
            int lo = (blk[6 + (i >> 1)] >> (4 * (i & 1))) & 15;
            int hi = (blk[2 + (i >> 3)] >> (i & 7)) & 1;
            out[b * 32 + i] = (float)((lo | (hi << 4)) - 16) * d;
        }
    }
}

/* Q5_1, 24 B: d @0, m @2, qh[4] @4, qs[16] @8; out = d*q + m (cpp/src/dequant.cpp:78-93). */
void vbo_dequantize_row_q5_1(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 32 < n; ++b) {
        const uint8_t* blk = row + b * 24;
        float d = vbo_f16_to_f32(rd16(blk)), m = vbo_f16_to_f32(rd16(blk + 2));
        for (int64_t i = 0; i < rem_of(n, b, 32); ++i) {
            int lo = (blk[8 + (i >> 1)] >> (4 * (i & 1))) & 15;
            int hi = (blk[4 + (i >> 3)] >> (i & 7)) & 1;
            float p = d * (float)(lo | (hi << 4));
            out[b * 32 + i] = p + m;
        }
    }
}

/* Q2_K, 84 B: scales[16] @0, qs[64] @16, d @80, dmin @82.  Value v: sub-block s = v>>4,
 * l = v&15; code = bits 2(l&3).. of qs[4s + (l>>3)] (so values l and l+4 of a half share a
 * code); out = (d*(scales[s]&15))*code + dmin -- the reference adds dmin itself, without
 * a per-sub-block min (cpp/src/dequant.cpp:128-150). */
void vbo_dequantize_row_q2_K(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 256 < n; ++b) {
        const uint8_t* blk = row + b * 84;
        float d = vbo_f16_to_f32(rd16(blk + 80)), mn = vbo_f16_to_f32(rd16(blk + 82));
        for (int64_t v = 0; v < rem_of(n, b, 256); ++v) {
            int s = (int)(v >> 4), l = (int)(v & 15);
            float dl = d * (float)(blk[s] & 15);
            int q = (blk[16 + 4 * s + (l >> 3)] >> (2 * (l & 3))) & 3;
            float p = dl * (float)q;
            out[b * 256 + v] = p + mn;
        }
    }
}

/* Q3_K scale of sub-block j (get_scale_min_k3, cpp/src/dequant.cpp:155-166; its min is
 * never used). */
static int q3k_scale(int j, const uint8_t* s) {
    if (j < 4) return s[j] & 63;
    if (j < 8) return s[j + 4] & 63;
    return (s[j - 4] >> 4) & 63;
}

/* Q3_K, 110 B: hmask[32] @0, qs[64] @32, scales[12] @96, d @108.  Value v: chunk c = v>>6,
 * quarter t = (v>>4)&3, l = v&15; code = bits 2(l&3).. of qs[16c + 4t + (l>>3)]; high bit =
 * bit (4c + 2t) of hmask[l], which is 0 once that shift reaches 8 (a byte shifted as an int);
 * out = (d*scale(4c + t))*(code + 8*high) (cpp/src/dequant.cpp:168-218). */
void vbo_dequantize_row_q3_K(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 256 < n; ++b) {
        const uint8_t* blk = row + b * 110;
        float d = vbo_f16_to_f32(rd16(blk + 108));
        for (int64_t v = 0; v < rem_of(n, b, 256); ++v) {
            int c = (int)(v >> 6), t = (int)((v >> 4) & 3), l = (int)(v & 15);
            float dt = d * (float)q3k_scale(4 * c + t, blk + 96);
            int q = (blk[32 + 16 * c + 4 * t + (l >> 3)] >> (2 * (l & 3))) & 3;
            int sh = 4 * c + 2 * t;
            int h = sh < 8 ? (blk[l] >> sh) & 1 : 0;
            out[b * 256 + v] = dt * (float)(q + 8 * h);
        }
    }
}

/* Q5_K, 176 B: d @0, dmin @2, scales[12] @4 (the Q4_K packing), qh[32] @16, qs[128] @48.
 * The reference steps its qh pointer by 32 bytes per 64-value chunk like qs, so chunk c
 * takes its fifth bits from bytes 16+32c.. (qs bytes from chunk 1 on) and always from bit
 * 7 (first half) or bit 3 (second half).  Value v: c = v>>6, half = (v>>5)&1, l = v&31;
 * out = (d*sc)*q - dmin*m with (sc, m) of sub-block 2c+half (cpp/src/dequant.cpp:307-354). */
void vbo_dequantize_row_q5_K(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 256 < n; ++b) {
        const uint8_t* blk = row + b * 176;
        float d = vbo_f16_to_f32(rd16(blk)), dmin = vbo_f16_to_f32(rd16(blk + 2));
        for (int64_t v = 0; v < rem_of(n, b, 256); ++v) {
            int c = (int)(v >> 6), half = (int)((v >> 5) & 1), l = (int)(v & 31);
            int sc, mn;
            q4k_scale_min(2 * c + half, blk + 4, &sc, &mn);
            float d1 = d * (float)sc, m1 = dmin * (float)mn;
            int qb = blk[48 + 32 * c + l], hb = blk[16 + 32 * c + l];
            int q = half ? ((qb >> 4) | (((hb >> 3) & 1) << 4)) : ((qb & 15) | (((hb >> 7) & 1) << 4));
            float p = d1 * (float)q;
            out[b * 256 + v] = p - m1;
        }
    }
}

/* Q8_K, 292 B: d (float32) @0, then eight 33-byte sub-blocks at 4 + 33s: 32 int8 codes and
 * an int8 scale; out = code * (d*scale) (cpp/src/dequant.cpp:226-245). */
void vbo_dequantize_row_q8_K(const uint8_t* row, float* out, int64_t n) {
    for (int64_t b = 0; b * 256 < n; ++b) {
        const uint8_t* blk = row + b * 292;
        float d;
        memcpy(&d, blk, 4);
        for (int64_t v = 0; v < rem_of(n, b, 256); ++v) {
            const uint8_t* sub = blk + 4 + 33 * (v >> 5);
            float ds = d * (float)(int8_t)sub[32];
            out[b * 256 + v] = (float)(int8_t)sub[v & 31] * ds;
        }
    }
}

/* Dispatcher (cpp/src/dequant.cpp:407-425).  Returns 0, or -1 for an unsupported type
 * where the reference throws "Unsupported dequant type". */
int vbo_dequantize_row(const void* row, float* out, int64_t n, int32_t type) {
    switch (type) {
        case VBO_F32: vbo_row_f32((const uint8_t*)row, out, n); return 0;
        case VBO_F16: vbo_row_f16((const uint8_t*)row, out, n); return 0;
        case VBO_BF16: vbo_row_bf16((const uint8_t*)row, out, n); return 0;
        case VBO_Q4_K: vbo_dequantize_row_q4_K((const uint8_t*)row, out, n); return 0;
        case VBO_Q6_K: vbo_dequantize_row_q6_K((const uint8_t*)row, out, n); return 0;
        case VBO_Q8_0: vbo_dequantize_row_q8_0((const uint8_t*)row, out, n); return 0;
        case VBO_Q4_0: vbo_dequantize_row_q4_0((const uint8_t*)row, out, n); return 0;
        case VBO_Q4_1: vbo_dequantize_row_q4_1((const uint8_t*)row, out, n); return 0;
        case VBO_Q5_0: vbo_dequantize_row_q5_0((const uint8_t*)row, out, n); return 0;
        case VBO_Q5_1: vbo_dequantize_row_q5_1((const uint8_t*)row, out, n); return 0;
        case VBO_Q2_K: vbo_dequantize_row_q2_K((const uint8_t*)row, out, n); return 0;
        case VBO_Q3_K: vbo_dequantize_row_q3_K((const uint8_t*)row, out, n); return 0;
        case VBO_Q5_K: vbo_dequantize_row_q5_K((const uint8_t*)row, out, n); return 0;
        case VBO_Q8_K: vbo_dequantize_row_q8_K((const uint8_t*)row, out, n); return 0;
        default: return -1;
    }
}

/* Dequantize `rows` rows of a K x N matrix (stride vbo_row_bytes). */
int vbo_dequantize_matrix(const void* w, float* out, int64_t rows, int64_t n, int32_t type) {
    int64_t rb = vbo_row_bytes(type, n);
    if (rb < 0) return -1;
    for (int64_t r = 0; r < rows; ++r)
        if (vbo_dequantize_row((const uint8_t*)w + r * rb, out + r * n, n, type)) return -1;
    return 0;
}

/* gemv_dequant (cpp/src/dequant.cpp:739-780): out[n] = sum_k x[k] * deq(W[k])[n],
 * W = K rows of N values (blocks along N), accumulated in fp32 sequentially in k:
 * zero out, then per row dequantize into scratch and out[n] += x[k]*scratch[n]. */
int vbo_gemv_dequant(const float* x, const void* w, float* out, int64_t K, int64_t N,
                     int32_t type, float* scratch) {
    int64_t rb = vbo_row_bytes(type, N);
    if (rb < 0) return -1;
    for (int64_t n = 0; n < N; ++n) out[n] = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
        if (vbo_dequantize_row((const uint8_t*)w + k * rb, scratch, N, type)) return -1;
        float xk = x[k];
        for (int64_t n = 0; n < N; ++n) {
            float p = xk * scratch[n];
            out[n] = out[n] + p;
        }
    }
    return 0;
}

/* Batched form: B independent gemv_dequant calls, x [B,K] -> out [B,N], which is how
 * the reference engine handles several tokens (one call per token,
 * cpp/src/fast_model.cpp:645-660). */
int vbo_gemv_dequant_batch(const float* x, const void* w, float* out, int64_t K, int64_t N,
                           int32_t type, int64_t batch) {
    float* scratch = (float*)malloc((size_t)N * sizeof(float));
    if (!scratch) return -2;
    int rc = 0;
    for (int64_t b = 0; b < batch && rc == 0; ++b)
        rc = vbo_gemv_dequant(x + b * K, w, out + b * N, K, N, type, scratch);
    free(scratch);
    return rc;
}

/* Wide-accumulator reference GEMM for checking the bf16 tensor-core path:
 * C[m,n] = sum_k A[m,k] * deq(W)[k,n] in double, A given as fp32 (the bf16 values
 * widened).  The reference has no batched GEMM; it loops gemv_dequant per token
 * (cpp/src/fast_model.cpp:645-660), so this is the exact sum that loop approximates. */
int vbo_gemm_f64(const float* a, const void* w, double* c, int64_t M, int64_t K, int64_t N,
                 int32_t type) {
    int64_t rb = vbo_row_bytes(type, N);
    if (rb < 0) return -1;
    float* row = (float*)malloc((size_t)N * sizeof(float));
    if (!row) return -2;
    for (int64_t i = 0; i < M * N; ++i) c[i] = 0.0;
    for (int64_t k = 0; k < K; ++k) {
        if (vbo_dequantize_row((const uint8_t*)w + k * rb, row, N, type)) { free(row); return -1; }
        for (int64_t m = 0; m < M; ++m) {
            double am = (double)a[m * K + k];
            if (am == 0.0) continue;
            double* cr = c + m * N;
            for (int64_t n = 0; n < N; ++n) cr[n] += am * (double)row[n];
        }
    }
    free(row);
    return 0;
}
