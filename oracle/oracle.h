/*
 * CPU oracle for the shlo_cuda hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker, never the product. Only the test suite
 * (tests/), __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its
 * `--impl reference` arm) may load it. The CUDA library never links it and no
 * product code path falls back to it.
 *
 * It restates, in plain C compiled with -ffp-contract=off, the arithmetic the
 * reference pins its GPU kernels to (ggml-cpu's arm64 NEON order, V-Sekai-fire/
 * ggml @29cae86, as the reference's Lean kernel specs spell it out):
 *   - splitmix32 / unif input streams            ref/ggml_ref.c:21-30, 38-43
 *   - ggml_v_expf, lane by lane                  StablehloMlx/Kernels/Math.lean:28-49
 *   - ggml_vec_dot_f32 (mul_mat) and both tails  StablehloMlx/Kernels/Shaders.lean:55-91
 *   - soft_max                                   Shaders.lean:100-123
 *   - norm                                       Shaders.lean:130-166
 *   - silu                                       Shaders.lean:172-179
 *   - gelu_erf                                   Shaders.lean:186-199 (erff: correctly rounded)
 *   - binary32 / and sqrt, binary64 soft float   StablehloMlx/Kernels/SoftFloat.lean:54-305
 * Row tails of soft_max and silu use a correctly rounded expf, the function the
 * pinned reference build links (CORE-MATH, ref/build.sh:52).
 *
 * Parity is pinned: tests regenerate every ggml_ref case's inputs and compare
 * the SHA-256 of the oracle's outputs with evidence/ref-{stock,pinned}.sha256
 * (copied to tests/golden/).
 */
#ifndef SHLO_ORACLE_H
#define SHLO_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_PINNED = 0, ORC_STOCK = 1 };

/* splitmix32 and the uniform stream of ref/ggml_ref.c:21-30. */
uint32_t orc_splitmix32(uint32_t *state);
void orc_unif(uint32_t *state, float a, float *out, size_t n);

float orc_ggml_v_expf(float x);
float orc_expf_cr(float x);
float orc_erff_cr(float x);

/* y[r*M+m] = ggml_vec_dot_f32(w + (r/N)*wbs + m*K, x + r*K); nthreads >= 1. */
void orc_mul_mat(const float *w, const float *x, float *y, int K, int M, int R, int N, long wbs,
                 int flavour, int nthreads);
void orc_soft_max(const float *x, float *y, int ncols, int rows, float scale, int nthreads);
void orc_norm(const float *x, float *y, int ncols, int rows, float eps, int nthreads);
void orc_silu(const float *x, float *y, int ncols, int rows);
void orc_gelu_erf(const float *x, float *y, size_t n, int nthreads);
void orc_erff_range(uint32_t base, uint32_t count, uint32_t *out, int nthreads);
float orc_scale(float x, float s);

/* The reference's soft-float semantics (SoftFloat.lean), as integer code. */
float orc_f32_div(float a, float b);
float orc_f32_sqrt(float a);
uint64_t orc_f64_from_f32(float x);
float orc_f64_to_f32(uint64_t d);
uint64_t orc_f64_add(uint64_t a, uint64_t b);
uint64_t orc_f64_sub(uint64_t a, uint64_t b);
uint64_t orc_f64_mul(uint64_t a, uint64_t b);
uint64_t orc_f64_div(uint64_t a, uint64_t b);
uint64_t orc_f64_floor(uint64_t a);
uint64_t orc_f64_to_i64(uint64_t a);
/* Elementwise forms over arrays (op codes as the f64_ew kernel: 0 add .. 5 to-int64). */
void orc_f64_ew(int op, const uint64_t *a, const uint64_t *b, uint64_t *y, size_t n);
void orc_f64_of_f32_arr(const float *a, uint64_t *y, size_t n);
void orc_f32_of_f64_arr(const uint64_t *a, float *y, size_t n);
void orc_f32_div_arr(const float *a, const float *b, float *y, size_t n);
void orc_f32_sqrt_arr(const float *a, float *y, size_t n);

#ifdef __cplusplus
}
#endif
#endif
