/*
 * synth.c — host restatement of the library's seeded synthetic-input
 * generator (SplitMix64 finaliser over a counter; fp16(RNE(U(0,0.01))) block
 * scales; Box-Muller normals).
 *
 * TEST INFRASTRUCTURE ONLY: lets the CPU legs of the benchmark and the tests
 * build a layer's bytes without loading the product library. Its output is
 * checked byte for byte against the product's own generator
 * (tests/test_synth.py). The generator is this project's definition of the
 * synthetic benchmark inputs, not reference code.
 */
#include <math.h>
#include <stdint.h>

#include "oracle.h"

static uint64_t fmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static uint64_t key_of(uint64_t seed, uint64_t stream) {
    return fmix64(seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull + 0x632BE59BD9B4E019ull);
}
static uint64_t word_of(uint64_t key, uint64_t i) { return fmix64(key + (i + 1) * 0x9E3779B97F4A7C15ull); }
static double unit_of(uint64_t w) { return (double)(w >> 11) * 0x1.0p-53; }

/* fp16 bits of v >= 0, round to nearest even */
static uint16_t half_rne(double v) {
    if (!(v > 0.0)) return 0;
    if (v < 0x1.0p-14) return (uint16_t)rint(v * 0x1.0p24);
    int e;
    double fr = frexp(v, &e);
    double mant = rint((fr * 2.0 - 1.0) * 1024.0);
    int ex = e - 1;
    if (mant >= 1024.0) { mant = 0.0; ex += 1; }
    if (ex > 15) return 0x7C00;
    return (uint16_t)(((ex + 15) << 10) | (int)mant);
}

static uint16_t scale_bits(uint64_t ks, uint64_t i) { return half_rne(unit_of(word_of(ks, i)) * 0.01); }

void orc_synth_blocks(void *dst, int type, uint64_t n_blocks, uint64_t first_block, uint64_t seed,
                      uint64_t stream_id) {
    const uint64_t kq = key_of(seed, 2 * stream_id), ks = key_of(seed, 2 * stream_id + 1);
    const int q4 = type == ORC_TYPE_Q4_K;
    const int bytes = q4 ? ORC_Q4K_BYTES : ORC_Q6K_BYTES, words = q4 ? 18 : 27;
    uint8_t *p = (uint8_t *)dst;
    for (uint64_t b = 0; b < n_blocks; b++) {
        const uint64_t gb = first_block + b;
        uint8_t *blk = p + b * bytes;
        for (int j = 0; j < words; j++) {
            uint64_t w = word_of(kq, gb * (uint64_t)words + j);
            if (q4 && j == 0)
                w = (w & ~0xFFFFFFFFull) | scale_bits(ks, 2 * gb) | ((uint64_t)scale_bits(ks, 2 * gb + 1) << 16);
            if (!q4 && j == 26) w = (w & ~0xFFFFull) | scale_bits(ks, gb);
            const int nb = (8 * j + 8 <= bytes) ? 8 : bytes - 8 * j;
            for (int k = 0; k < nb; k++) blk[8 * j + k] = (uint8_t)(w >> (8 * k));
        }
    }
}

void orc_synth_normal(float *dst, uint64_t n, uint64_t seed, uint64_t stream_id, float sigma) {
    const uint64_t k = key_of(seed, 0x4E4F524Dull ^ (stream_id << 1));
    for (uint64_t i = 0; i < n; i++) {
        const double u1 = 1.0 - unit_of(word_of(k, 2 * i));
        const double u2 = unit_of(word_of(k, 2 * i + 1));
        dst[i] = (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2) * (double)sigma);
    }
}
