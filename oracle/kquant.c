/*
 * kquant.c — CPU restatement of ornith-flight's Q4_K / Q6_K super-block decode.
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker, never the product.
 *
 * Block layouts (engine/src/third_party/gguf.h:27-40):
 *   Q4_K, 144 B: u16 d, u16 dmin, u8 scales[12], u8 qs[128]
 *   Q6_K, 210 B: u8 ql[128], u8 qh[64], i8 scales[16], u16 d
 * Values are read byte-wise (little-endian), so no struct packing is assumed.
 */
#include "oracle.h"
#include <string.h>

static uint16_t rd_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* engine/src/gguf.c:16-26 — not IEEE: only 0x0000 is special-cased; every
 * other pattern (subnormals, -0, exponent 31) is rebiased as if normal. */
float orc_fp16_to_fp32(uint16_t h) {
    if (h == 0) return 0.0f;
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t expo = (((uint32_t)h >> 10) & 0x1Fu) + 112u;
    uint32_t mant = (uint32_t)(h & 0x3FFu) << 13;
    uint32_t bits = sign | (expo << 23) | mant;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* engine/src/gguf.c:31-40 — 6-bit (scale, min) of sub-block j (0..7). */
static void q4k_scale_min(const uint8_t *s, int j, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 0x3F;
        *mn = s[j + 4] & 0x3F;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* One Q4_K element. Arithmetic follows gguf.c:49-57 / :521-527:
 * y = (d*sc)*q - (dmin*m), each product rounded separately. */
static float q4k_elem(float d, float dmin, const uint8_t *scales, const uint8_t *qs, int pos) {
    int chunk = pos >> 6;        /* 64-element chunk: 32 qs bytes */
    int hi = (pos >> 5) & 1;     /* low nibbles first, then high nibbles */
    int sub = 2 * chunk + hi;
    int sc, mn;
    q4k_scale_min(scales, sub, &sc, &mn);
    uint8_t byte = qs[chunk * 32 + (pos & 31)];
    int q = hi ? (byte >> 4) : (byte & 0x0F);
    float dsc = d * (float)sc;
    float mm = dmin * (float)mn;
    return dsc * (float)q - mm;
}

/* engine/src/gguf.c:43-61 */
void orc_q4k_block(const uint8_t *blk, float *y) {
    float d = orc_fp16_to_fp32(rd_u16(blk));
    float dmin = orc_fp16_to_fp32(rd_u16(blk + 2));
    for (int p = 0; p < ORC_QK; p++) y[p] = q4k_elem(d, dmin, blk + 4, blk + 16, p);
}

/* engine/src/gguf.c:511-528 */
float orc_q4k_one(const uint8_t *blk, int pos) {
    float d = orc_fp16_to_fp32(rd_u16(blk));
    float dmin = orc_fp16_to_fp32(rd_u16(blk + 2));
    return q4k_elem(d, dmin, blk + 4, blk + 16, pos);
}

/* One Q6_K element; engine/src/gguf.c:64-86 and :532-571.
 * pos = 128*half + 32*quad + l; quad selects (ql byte +0/+32, nibble lo/hi,
 * qh bit pair), scale index = 8*half + 2*quad + l/16. y = (d*sc)*q. */
static float q6k_elem(const uint8_t *blk, int pos) {
    const uint8_t *ql = blk;
    const uint8_t *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    float d = orc_fp16_to_fp32(rd_u16(blk + 208));
    int half = pos >> 7;
    int quad = (pos >> 5) & 3;
    int l = pos & 31;
    uint8_t lo_byte = ql[half * 64 + (quad & 1) * 32 + l];
    int nib = (quad < 2) ? (lo_byte & 0x0F) : (lo_byte >> 4);
    int top = (qh[half * 32 + l] >> (2 * quad)) & 3;
    int q = (nib | (top << 4)) - 32;
    int s = sc[half * 8 + quad * 2 + (l >> 4)];
    float ds = d * (float)s;
    return ds * (float)q;
}

void orc_q6k_block(const uint8_t *blk, float *y) {
    for (int p = 0; p < ORC_QK; p++) y[p] = q6k_elem(blk, p);
}

float orc_q6k_one(const uint8_t *blk, int pos) { return q6k_elem(blk, pos); }

/* engine/src/gguf.c:605-638 */
int orc_dequant_tensor(const void *data, int type, uint64_t n_elems, float *out) {
    if (!data || !out) return 0;
    const uint8_t *b = (const uint8_t *)data;
    uint64_t nb = n_elems / ORC_QK;
    switch (type) {
    case ORC_TYPE_F32:
        memcpy(out, data, n_elems * 4);
        return 1;
    case ORC_TYPE_F16:
        for (uint64_t i = 0; i < n_elems; i++) out[i] = orc_fp16_to_fp32(rd_u16(b + 2 * i));
        return 1;
    case ORC_TYPE_Q4_K:
        for (uint64_t i = 0; i < nb; i++) orc_q4k_block(b + i * ORC_Q4K_BYTES, out + i * ORC_QK);
        return 1;
    case ORC_TYPE_Q6_K:
        for (uint64_t i = 0; i < nb; i++) orc_q6k_block(b + i * ORC_Q6K_BYTES, out + i * ORC_QK);
        return 1;
    default:
        return 0;
    }
}

/* engine/src/gguf.c:652-711 — element i of expert e is linear element i*E+e. */
int orc_dequant_slice(const void *data, int type, uint64_t n_elems,
                      uint64_t n_experts, int expert, float *out) {
    if (!data || !out || expert < 0 || n_experts == 0) return 0;
    if ((uint64_t)expert >= n_experts) return 0;
    const uint8_t *b = (const uint8_t *)data;
    uint64_t per = n_elems / n_experts;
    for (uint64_t i = 0; i < per; i++) {
        uint64_t lin = i * n_experts + (uint64_t)expert;
        switch (type) {
        case ORC_TYPE_F32: memcpy(&out[i], b + 4 * lin, 4); break;
        case ORC_TYPE_F16: out[i] = orc_fp16_to_fp32(rd_u16(b + 2 * lin)); break;
        case ORC_TYPE_Q4_K:
            out[i] = orc_q4k_one(b + (lin / ORC_QK) * ORC_Q4K_BYTES, (int)(lin % ORC_QK));
            break;
        case ORC_TYPE_Q6_K:
            out[i] = orc_q6k_one(b + (lin / ORC_QK) * ORC_Q6K_BYTES, (int)(lin % ORC_QK));
            break;
        default: return 0;
        }
    }
    return 1;
}
