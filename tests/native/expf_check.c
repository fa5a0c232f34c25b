/* Exhaustive host check of exact_expf.h: its formula (compiled here as host C)
 * must equal this host C library's expf for every float x <= 0.
 * Prints the number of mismatches and exits non-zero if any. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "exact_expf.h"

int main(void) {
    long bad = 0;
    /* +0, then every pattern with the sign bit set up to -inf (NaNs excluded) */
#pragma omp parallel for reduction(+ : bad) schedule(static, 1 << 20)
    for (int64_t b = 0x7FFFFFFFLL; b <= 0xFF800000LL; b++) {
        uint32_t bits = (b == 0x7FFFFFFFLL) ? 0u : (uint32_t)b;
        float x;
        memcpy(&x, &bits, 4);
        float want = expf(x), got = ofb_exact_expf(x);
        if (memcmp(&want, &got, 4) != 0) bad++;
    }
    printf("%ld\n", bad);
    return bad != 0;
}
