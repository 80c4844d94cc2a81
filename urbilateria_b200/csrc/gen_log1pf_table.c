/*
 * gen_log1pf_table.c — build step: records where this system's libm `log1pf` (the function
 * Rust's f32::ln_1p calls on x86_64-linux-gnu, used by DeepSeek-V4's router softplus,
 * src/models/deepseek_v4/math.rs:604-610) differs from a single rounding of the
 * double-precision log1p, over the softplus argument range [0, 1].
 *
 * The device evaluates log1pf(x) as (float)log1p((double)x).  That equals libm log1pf except
 * for (a) inputs where libm is not correctly rounded and (b) inputs whose exact log1p lies so
 * close to a float rounding midpoint that a double log1p with <= 1 ulp error could round
 * either way.  Both sets are written, with libm's result, as sorted (input bits, output bits)
 * uint32 little-endian pairs; the library embeds the table.
 *
 * Usage: gen_log1pf_table OUT.bin     (OpenMP)
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t to_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* 1 when the long-double value is within 2^-48 (relative) of the midpoint next to f. */
static int near_midpoint(long double e, float f) {
    if (!isfinite(f) || f == 0.0f) return 0;
    float up = nextafterf(f, INFINITY), dn = nextafterf(f, 0.0f);
    long double mid_up = ((long double)f + (long double)up) / 2.0L;
    long double mid_dn = ((long double)f + (long double)dn) / 2.0L;
    long double tol = fabsl(e) * 0x1p-48L;
    return fabsl(e - mid_up) < tol || fabsl(e - mid_dn) < tol;
}

int main(int argc, char **argv) {
    if (argc != 2) { fprintf(stderr, "usage: %s OUT.bin\n", argv[0]); return 2; }
    const int64_t n = (int64_t)0x3F800000 + 1;  /* +0.0 .. 1.0 */
    const int chunks = 1024;
    uint32_t **keys = calloc(chunks, sizeof(uint32_t *));
    uint32_t **vals = calloc(chunks, sizeof(uint32_t *));
    int64_t *counts = calloc(chunks, sizeof(int64_t));
#pragma omp parallel for schedule(dynamic, 1)
    for (int c = 0; c < chunks; ++c) {
        int64_t begin = n * c / chunks, end = n * (c + 1) / chunks, cap = 1024, used = 0;
        uint32_t *k = malloc(cap * 4), *v = malloc(cap * 4);
        for (int64_t i = begin; i < end; ++i) {
            float x = from_bits((uint32_t)i);
            float lib = log1pf(x);
            float dbl = (float)log1p((double)x);
            long double e = log1pl((long double)x);
            int exception = to_bits(lib) != to_bits(dbl) || near_midpoint(e, dbl);
            if (!exception) continue;
            if (used == cap) { cap *= 2; k = realloc(k, cap * 4); v = realloc(v, cap * 4); }
            k[used] = (uint32_t)i;
            v[used] = to_bits(lib);
            ++used;
        }
        keys[c] = k; vals[c] = v; counts[c] = used;
    }
    FILE *out = fopen(argv[1], "wb");
    if (!out) { perror("fopen"); return 1; }
    int64_t total = 0;
    for (int c = 0; c < chunks; ++c) {
        for (int64_t i = 0; i < counts[c]; ++i) {
            uint32_t pair[2] = {keys[c][i], vals[c][i]};
            fwrite(pair, 4, 2, out);
        }
        total += counts[c];
    }
    fclose(out);
    fprintf(stderr, "log1pf exception table: %lld entries\n", (long long)total);
    return 0;
}
