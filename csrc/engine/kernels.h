// FP4 row-dot kernels of the CPU expert engine, one set per ISA, chosen once per process (engine.cpp).
//
// A kernel computes out[r * n + t] = sum_k w_r[k] * x_t[k] for `rows` FP4 rows (E2M1 codes, low nibble first, block
// scales applied, global scales not) against n <= MAX_TOK prepared token vectors. Token vectors are prepared once per
// call in the kernel's own layout (prep_x from BF16, prep_mid from FP32), so the inner loop does no shuffling:
//   avx512: BF16, each 64-element chunk split into its 32 even then 32 odd elements; a "hilo" vector is the exact
//           BF16 pair hi + lo of an FP32 vector (hi chunk layout for all K, then lo), used by the down projection so
//           the FP32 intermediate is not rounded to BF16.
//   avx2:   FP32, each 16-element chunk split into its 8 even then 8 odd elements.
//   scalar: FP32 in order.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace xt {

constexpr int MAX_TOK = 8;   // tokens per micro-group: register blocking of the kernels

enum Fmt { NVFP4 = 0, MXFP4 = 1 };

struct Kernels {
    const char *name;
    int chunk;                 // K must be a multiple of this
    size_t x_bytes_per_elem;   // prepared activation bytes per element (hilo: twice)
    size_t mid_bytes_per_elem;
    void (*prep_x)(const uint16_t *x, int K, void *dst);
    // write element j of an FP32 vector into its prepared slot (used by the gate/up tasks on their own rows)
    void (*store_mid)(void *dst, int K, int j, float v);
    void (*dot)(const uint8_t *w, size_t wstride, const uint8_t *s, size_t sstride, int rows, int K, int fmt,
                const void *const *xs, int n, int mid, float *out);
};

const Kernels *kernels_avx512();   // NULL when the CPU lacks AVX-512 BF16
const Kernels *kernels_avx2();     // NULL without AVX2/FMA
const Kernels *kernels_scalar();

float e4m3_value(uint8_t b);
float ue8m0_value(uint8_t b);

}  // namespace xt
