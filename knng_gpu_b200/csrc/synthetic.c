/*
 * synthetic.c -- seeded synthetic datasets for the benchmark configurations
 * and the dataset hash (host C, libknng_synth.so). Every dataset is drawn row-major from one
 * knng::random::XorShift64 stream (include/knng/random.hpp:48-144): the
 * (13, 7, 17) xorshift, next_float01 = top 24 bits / 2^24, next_below =
 * Lemire multiply-high, as in the reference's bench generator
 * (benchmarks/bench_brute_force.cpp:57-68).
 *
 * Recipes (kind):
 *   0  uniform integers:   x = (float) next_below(256)
 *   1  Gaussian mixture:   `components` centres, each coordinate
 *                          2*next_float01()-1 (all centres first); then per
 *                          point c = next_below(components) and per
 *                          coordinate x = centre + sigma * z, z standard
 *                          normal by Box-Muller on two next_float01() draws:
 *                          z = sqrt(-2 ln(1-u1)) * cos(2 pi u2) in double,
 *                          rounded to float once.
 *   2  unit rows:          x = next_float01(), then every row divided by
 *                          sqrtf of its sequential fp32 sum of squares
 *   3  sparse integers:    next_float01() < p_zero ? 0 : 1 + next_below(255)
 *   4  uniform [-1, 1):    2*next_float01()-1 (the reference bench's data)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

static uint64_t xs_next(uint64_t *s)
{
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return x;
}

static float xs_float01(uint64_t *s)
{
    const uint64_t bits = (xs_next(s) >> 40) & ((1ull << 24) - 1);
    return (float)bits * (1.0f / (float)(1u << 24));
}

static uint64_t xs_below(uint64_t *s, uint64_t bound)
{
    if (bound <= 1) return 0;
    const unsigned __int128 p = (unsigned __int128)xs_next(s) * bound;
    return (uint64_t)(p >> 64);
}

/* One row of recipe `kind` from the stream `s` (kinds 0, 2, 3, 4; kind 1
 * with its centres in `centres`). */
static void gen_row(int kind, uint64_t *s, uint64_t d, float *row, const float *centres, uint64_t components,
                    float sigma, float p_zero)
{
    switch (kind) {
    case 0:
        for (uint64_t j = 0; j < d; ++j) row[j] = (float)xs_below(s, 256);
        break;
    case 1: {
        const double two_pi = 6.283185307179586476925286766559;
        const float *c = centres + xs_below(s, components) * d;
        for (uint64_t j = 0; j < d; ++j) {
            const double u1 = (double)xs_float01(s);
            const double u2 = (double)xs_float01(s);
            const float z = (float)(sqrt(-2.0 * log(1.0 - u1)) * cos(two_pi * u2));
            row[j] = c[j] + sigma * z;
        }
        break;
    }
    case 2: {
        float acc = 0.0f;
        for (uint64_t j = 0; j < d; ++j) {
            row[j] = xs_float01(s);
            const float sq = row[j] * row[j];
            acc = acc + sq;
        }
        const float norm = sqrtf(acc);
        if (norm > 0.0f)
            for (uint64_t j = 0; j < d; ++j) row[j] = row[j] / norm;
        break;
    }
    case 3:
        for (uint64_t j = 0; j < d; ++j) row[j] = xs_float01(s) < p_zero ? 0.0f : (float)(1 + xs_below(s, 255));
        break;
    default: /* 4 */
        for (uint64_t j = 0; j < d; ++j) row[j] = 2.0f * xs_float01(s) - 1.0f;
        break;
    }
}

/* Rows [row_begin, row_begin + row_count) of the dataset of `kind` (the
 * same values as the full dataset holds there; the stream is advanced over
 * the rows before). Returns 0 on success, -1 for an unknown kind, a zero
 * seed or missing scratch. `scratch` must hold components*d floats for kind
 * 1 plus d floats (d floats for the other kinds; may be NULL when
 * row_begin == 0 and kind != 1). */
int knng_synth_generate_rows(int kind, uint64_t seed, uint64_t row_begin, uint64_t row_count, uint64_t d, float *out,
                             uint64_t components, float sigma, float p_zero, float *scratch)
{
    if (seed == 0 || kind < 0 || kind > 4) return -1;
    if ((kind == 1 && (!scratch || components == 0)) || (row_begin > 0 && !scratch)) return -1;
    uint64_t s = seed;
    const float *centres = NULL;
    float *skip_row = scratch;
    if (kind == 1) {
        for (uint64_t i = 0; i < components * d; ++i) scratch[i] = 2.0f * xs_float01(&s) - 1.0f;
        centres = scratch;
        skip_row = scratch + components * d;
    }
    for (uint64_t r = 0; r < row_begin; ++r) gen_row(kind, &s, d, skip_row, centres, components, sigma, p_zero);
    for (uint64_t r = 0; r < row_count; ++r) gen_row(kind, &s, d, out + r * d, centres, components, sigma, p_zero);
    return 0;
}

/* Returns 0 on success, -1 for an unknown kind or a zero seed. `scratch`
 * must hold components*d floats for kind 1 (may be NULL otherwise). */
int knng_synth_generate(int kind, uint64_t seed, uint64_t n, uint64_t d, float *out, uint64_t components,
                        float sigma, float p_zero, float *scratch)
{
    if (kind == 1 && (!scratch || components == 0)) return -1;
    return knng_synth_generate_rows(kind, seed, 0, n, d, out, components, sigma, p_zero, scratch);
}

/* Sorted, distinct query ids for the subset harness: ids drawn with
 * next_below(n), repeats rejected, until `count` distinct ids are held;
 * returned in ascending order. */
int knng_synth_sample_ids(uint64_t seed, uint64_t n, uint64_t count, uint64_t *out)
{
    if (seed == 0 || count > n) return -1;
    const uint64_t words = (n + 63) / 64;
    uint64_t *bits = (uint64_t *)calloc(words, sizeof(uint64_t));
    if (!bits) return -1;
    uint64_t s = seed, got = 0;
    while (got < count) {
        const uint64_t v = xs_below(&s, n);
        if (bits[v >> 6] & (1ull << (v & 63))) continue;
        bits[v >> 6] |= 1ull << (v & 63);
        ++got;
    }
    uint64_t w = 0;
    for (uint64_t i = 0; i < n && w < count; ++i)
        if (bits[i >> 6] & (1ull << (i & 63))) out[w++] = i;
    free(bits);
    return 0;
}

/* FNV-1a 64 dataset hash over (u64 n, u64 d, fp32 payload): the key of the
 * ground-truth cache (src/bench/ground_truth.cpp:45-56, 90-101). */
uint64_t knng_dataset_hash(const float *x, uint64_t n, uint64_t d)
{
    uint64_t s = 14695981039346656037ull;
    const unsigned char *p;
    p = (const unsigned char *)&n;
    for (int i = 0; i < 8; ++i) { s ^= p[i]; s *= 1099511628211ull; }
    p = (const unsigned char *)&d;
    for (int i = 0; i < 8; ++i) { s ^= p[i]; s *= 1099511628211ull; }
    p = (const unsigned char *)x;
    for (uint64_t i = 0; i < n * d * 4; ++i) { s ^= p[i]; s *= 1099511628211ull; }
    return s;
}
