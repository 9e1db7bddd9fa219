/*
 * CPU oracle for the shlo_cuda hot path -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no fast-math, SSE2 floats).
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <quadmath.h>
#include <stdlib.h>
#include <string.h>

static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
/* arm64's default NaN: what an invalid operation (inf*0, inf-inf, 0/0) gives on
   the reference's CPU (x86 would give 0xFFC00000). Results of the reductions
   that are NaN are reported as this value. */
static inline float arm_nan(float v) { return v != v ? bitsf(0x7FC00000u) : v; }

/* ---- input streams: ref/ggml_ref.c:21-30 ---------------------------------- */

uint32_t orc_splitmix32(uint32_t *state) {
	uint32_t z = (*state += 0x9e3779b9u);
	z = (z ^ (z >> 16)) * 0x85ebca6bu;
	z = (z ^ (z >> 13)) * 0xc2b2ae35u;
	return z ^ (z >> 16);
}

void orc_unif(uint32_t *state, float a, float *out, size_t n) {
	for (size_t i = 0; i < n; i++)
		out[i] = a * ((float)(orc_splitmix32(state) >> 8) * (1.0f / 8388608.0f) - 1.0f);
}

/* ---- ggml_v_expf, one lane: StablehloMlx/Kernels/Math.lean:28-49 ------------
 * vfmaq_f32(a, b, c) = fmaf(b, c, a); vfmsq_f32(a, b, c) = fmaf(-b, c, a). */
float orc_ggml_v_expf(float x) {
	const float r = bitsf(0x4B400000);
	float z = fmaf(x, bitsf(0x3FB8AA3B), r);
	float n = z - r;
	float b = fmaf(-n, bitsf(0x35BFBE8E), fmaf(-n, bitsf(0x3F317200), x));
	uint32_t e = fbits(z) << 23;
	float k = bitsf(e + 0x3F800000u);
	float u = b * b;
	float p1 = fmaf(bitsf(0x3E2AAF33), b, bitsf(0x3EFFFEDB));
	float p2 = fmaf(bitsf(0x3C072010), b, bitsf(0x3D2B9F17));
	float p3 = fmaf(p2, u, p1);
	float j = fmaf(p3, u, bitsf(0x3F7FFFF6) * b);
	float an = fabsf(n);
	uint32_t d = (n <= 0.0f) ? 0x82000000u : 0u;
	float s1 = bitsf(d + 0x7F000000u);
	if (an > bitsf(0x43400000)) return s1 * s1;
	if (an > bitsf(0x42FC0000)) {
		float s2 = bitsf(e - d);
		return fmaf(s2, j, s2) * s1;
	}
	return fmaf(k, j, k);
}

/* ---- correct rounding to binary32 ----------------------------------------------
 * `y` approximates the exact value v with |y - v| <= |y| * 2^-rel_log2. Returns 1
 * and the correctly rounded float when no rounding boundary lies within that
 * bound, else 0. */
static int round_if_certain(long double y, int rel_log2, float *out) {
	float f = (float)y;
	long double tol = fabsl(y) * ldexpl(1.0L, -rel_log2);
	long double bounds[2];
	float lo = nextafterf(f, -INFINITY), hi = nextafterf(f, INFINITY);
	const long double top = (long double)FLT_MAX + ldexpl(1.0L, 103); /* the overflow boundary */
	bounds[0] = isinf(f) ? (f > 0 ? top : -top) : (isinf(lo) ? -top : ((long double)f + lo) / 2);
	bounds[1] = isinf(f) ? (f > 0 ? top : -top) : (isinf(hi) ? top : ((long double)f + hi) / 2);
	for (int i = 0; i < 2; i++)
		if (fabsl(y - bounds[i]) <= tol) return 0;
	*out = f;
	return 1;
}

static float round_quad_certain(__float128 y) {
	/* Quad results are within a few ulps (2^-110 relative); a binary32 value of a
	   transcendental function at a nonzero float is never that close to a midpoint. */
	float f = (float)y;
	__float128 lo = nextafterf(f, -INFINITY), hi = nextafterf(f, INFINITY);
	__float128 tol = fabsq(y) * 0x1p-104Q;
	if (!isinf(f) && ((!isinf((float)lo) && fabsq(y - ((__float128)f + lo) / 2) <= tol) ||
	                  (!isinf((float)hi) && fabsq(y - ((__float128)f + hi) / 2) <= tol)))
		abort();
	return f;
}

/* Correctly rounded erff. erf(-0) = -0; NaN returns the input quieted (what an
   arm64 libm returns: x + x). */
float orc_erff_cr(float x) {
	uint32_t b = fbits(x);
	if ((b & 0x7FFFFFFFu) > 0x7F800000u) return bitsf(b | 0x00400000u);
	if ((b & 0x7FFFFFFFu) == 0) return x;
	if ((b & 0x7FFFFFFFu) == 0x7F800000u) return (b >> 31) ? -1.0f : 1.0f;
	float f;
	if (round_if_certain(erfl((long double)x), 58, &f)) return f;
	return round_quad_certain(erfq((__float128)x));
}

/* Correctly rounded expf (the pinned build's CORE-MATH expf is correctly rounded). */
float orc_expf_cr(float x) {
	uint32_t b = fbits(x);
	if ((b & 0x7FFFFFFFu) > 0x7F800000u) return bitsf(b | 0x00400000u);
	if (b == 0x7F800000u) return x;
	if (b == 0xFF800000u) return 0.0f;
	if ((b & 0x7FFFFFFFu) == 0) return 1.0f;
	float f;
	if (round_if_certain(expl((long double)x), 58, &f)) return f;
	return round_quad_certain(expq((__float128)x));
}

/* ---- a tiny row-parallel helper ---------------------------------------------- */

typedef void (*rows_fn)(void *ctx, long r0, long r1);
struct rows_job { rows_fn fn; void *ctx; long r0, r1; };
static void *rows_thread(void *p) {
	struct rows_job *j = (struct rows_job *)p;
	j->fn(j->ctx, j->r0, j->r1);
	return NULL;
}
static void parallel_rows(rows_fn fn, void *ctx, long rows, int nthreads) {
	if (nthreads <= 1 || rows < 2) { fn(ctx, 0, rows); return; }
	if (nthreads > 256) nthreads = 256;
	if (nthreads > rows) nthreads = (int)rows;
	pthread_t th[256];
	struct rows_job jobs[256];
	for (int t = 0; t < nthreads; t++) {
		jobs[t].fn = fn; jobs[t].ctx = ctx;
		jobs[t].r0 = rows * t / nthreads; jobs[t].r1 = rows * (t + 1) / nthreads;
		pthread_create(&th[t], NULL, rows_thread, &jobs[t]);
	}
	for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* ---- mul_mat: ggml_vec_dot_f32, Shaders.lean:55-91 -------------------------
 * Sixteen accumulators a[j] (j = k mod 16) over blocks of 16 with fused
 * multiply-add, the GGML_F32x4_REDUCE tree, vaddvq_f32, then the tail:
 *   pinned: sumf = sumf + (w*x), two roundings (-ffp-contract=off);
 *   stock:  with a tail of 4 or more, its first (tail & ~3) elements add
 *           separate products in order, the rest use fmaf; a tail of 1-3 is fmaf. */
static float dot_ggml(const float *w, const float *x, int K, int flavour) {
	float a[16];
	for (int j = 0; j < 16; j++) a[j] = 0.0f;
	int np = K & ~15;
	for (int i = 0; i < np; i += 16)
		for (int j = 0; j < 16; j++) a[j] = fmaf(w[i + j], x[i + j], a[j]);
	for (int l = 0; l < 4; l++) a[l] = a[l] + a[8 + l];
	for (int l = 0; l < 4; l++) a[4 + l] = a[4 + l] + a[12 + l];
	for (int l = 0; l < 4; l++) a[l] = a[l] + a[4 + l];
	float sumf = (a[0] + a[1]) + (a[2] + a[3]);
	int tl = K - np;
	if (flavour == ORC_PINNED) {
		for (int i = np; i < K; i++) { float p = w[i] * x[i]; sumf = sumf + p; }
	} else {
		int nq = tl >= 4 ? (tl & ~3) : 0;
		for (int i = np; i < np + nq; i++) { float p = w[i] * x[i]; sumf = sumf + p; }
		for (int i = np + nq; i < K; i++) sumf = fmaf(w[i], x[i], sumf);
	}
	return sumf;
}

struct mm_ctx { const float *w, *x; float *y; int K, M, N, flavour; long wbs; };
static void mm_rows(void *p, long r0, long r1) {
	struct mm_ctx *c = (struct mm_ctx *)p;
	for (long r = r0; r < r1; r++) {
		const float *wb = c->w + (r / c->N) * c->wbs;
		const float *xr = c->x + r * (long)c->K;
		for (int m = 0; m < c->M; m++)
			c->y[r * (long)c->M + m] = arm_nan(dot_ggml(wb + (long)m * c->K, xr, c->K, c->flavour));
	}
}

void orc_mul_mat(const float *w, const float *x, float *y, int K, int M, int R, int N, long wbs,
                 int flavour, int nthreads) {
	struct mm_ctx c = { w, x, y, K, M, N, flavour, wbs };
	parallel_rows(mm_rows, &c, R, nthreads);
}

/* ---- soft_max: Shaders.lean:100-123 (ggml_compute_forward_soft_max_f32 with
 * ggml_vec_soft_max_f32). The row's last ncols mod 4 elements take the
 * correctly rounded expf, as the pinned build computes them. */
struct sm_ctx { const float *x; float *y; int n; float scale; };
static void sm_rows(void *p, long r0, long r1) {
	struct sm_ctx *c = (struct sm_ctx *)p;
	int n = c->n;
	float *wv = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
	for (long r = r0; r < r1; r++) {
		const float *x = c->x + r * (long)n;
		float *y = c->y + r * (long)n;
		float mx = -INFINITY;
		for (int i = 0; i < n; i++) {
			wv[i] = x[i] * c->scale;
			mx = (mx > wv[i]) ? mx : wv[i];
		}
		double sum = 0.0;
		int i = 0;
		for (; i + 3 < n; i += 4) {
			float e0 = orc_ggml_v_expf(wv[i] - mx), e1 = orc_ggml_v_expf(wv[i + 1] - mx);
			float e2 = orc_ggml_v_expf(wv[i + 2] - mx), e3 = orc_ggml_v_expf(wv[i + 3] - mx);
			y[i] = e0; y[i + 1] = e1; y[i + 2] = e2; y[i + 3] = e3;
			sum += (double)((e0 + e1) + (e2 + e3));
		}
		for (; i < n; i++) {
			float v = orc_expf_cr(wv[i] - mx);
			sum += (double)v;
			y[i] = v;
		}
		float inv = (float)(1.0 / sum);
		for (int k = 0; k < n; k++) y[k] = arm_nan(y[k] * inv);
	}
	free(wv);
}
void orc_soft_max(const float *x, float *y, int ncols, int rows, float scale, int nthreads) {
	struct sm_ctx c = { x, y, ncols, scale };
	parallel_rows(sm_rows, &c, rows, nthreads);
}

/* ---- norm: Shaders.lean:130-166 (ggml_compute_forward_norm_f32 without
 * Accelerate: ggml_vec_sum_f32, ggml_vec_cvar_f32, 1.0f/sqrtf(var + eps)). */
struct nm_ctx { const float *x; float *y; int n; float eps; };
static void nm_rows(void *p, long r0, long r1) {
	struct nm_ctx *c = (struct nm_ctx *)p;
	int n = c->n;
	for (long r = r0; r < r1; r++) {
		const float *x = c->x + r * (long)n;
		float *y = c->y + r * (long)n;
		double sum = 0.0;
		for (int i = 0; i < n; i++) sum += (double)x[i];
		float mean = (float)sum / (float)n;
		double s2 = 0.0;
		int i = 0;
		for (; i + 3 < n; i += 4) {
			float d0 = x[i] - mean, d1 = x[i + 1] - mean, d2 = x[i + 2] - mean, d3 = x[i + 3] - mean;
			float q0 = d0 * d0, q1 = d1 * d1, q2 = d2 * d2, q3 = d3 * d3;
			s2 += (double)((q0 + q1) + (q2 + q3));
		}
		for (; i < n; i++) { float d = x[i] - mean; float q = d * d; s2 += (double)q; }
		float var = (float)(s2 / (double)n);
		float scl = 1.0f / sqrtf(var + c->eps);
		for (int k = 0; k < n; k++) y[k] = arm_nan((x[k] - mean) * scl);
	}
}
void orc_norm(const float *x, float *y, int ncols, int rows, float eps, int nthreads) {
	struct nm_ctx c = { x, y, ncols, eps };
	parallel_rows(nm_rows, &c, rows, nthreads);
}

/* ---- silu: Shaders.lean:172-179 (ggml_vec_silu_f32: x / (1 + ggml_v_expf(0 - x))
 * on the four-lane body of each row; the row tail is x / (1 + expf(-x)) with
 * the correctly rounded expf). */
/* arm64's NaN rules for silu: a NaN input passes through every step quieted;
   an invalid division (-inf / inf) gives the default NaN. */
static float silu_nan(float x, float r) {
	uint32_t b = fbits(x);
	if ((b & 0x7FFFFFFFu) > 0x7F800000u) return bitsf(b | 0x00400000u);
	return arm_nan(r);
}
void orc_silu(const float *x, float *y, int ncols, int rows) {
	for (long r = 0; r < rows; r++) {
		const float *xr = x + r * (long)ncols;
		float *yr = y + r * (long)ncols;
		int i = 0;
		for (; i + 3 < ncols; i += 4)
			for (int l = 0; l < 4; l++) yr[i + l] = silu_nan(xr[i + l], xr[i + l] / (1.0f + orc_ggml_v_expf(0.0f - xr[i + l])));
		for (; i < ncols; i++) yr[i] = silu_nan(xr[i], xr[i] / (1.0f + orc_expf_cr(-xr[i])));
	}
}

/* ---- gelu_erf: Shaders.lean:186-199 (ggml_vec_gelu_erf_f32) ----------------- */
static float gelu_one(float x) {
	uint32_t b = fbits(x);
	if ((b & 0x7FFFFFFFu) > 0x7F800000u) return bitsf(b | 0x00400000u);
	return arm_nan((0.5f * x) * (1.0f + orc_erff_cr(x * bitsf(0x3F3504F3))));
}
struct ge_ctx { const float *x; float *y; };
static void ge_rows(void *p, long r0, long r1) {
	struct ge_ctx *c = (struct ge_ctx *)p;
	for (long i = r0; i < r1; i++) c->y[i] = gelu_one(c->x[i]);
}
void orc_gelu_erf(const float *x, float *y, size_t n, int nthreads) {
	struct ge_ctx c = { x, y };
	parallel_rows(ge_rows, &c, (long)n, nthreads);
}

struct ef_ctx { uint32_t base; uint32_t *out; };
static void ef_rows(void *p, long r0, long r1) {
	struct ef_ctx *c = (struct ef_ctx *)p;
	for (long i = r0; i < r1; i++) c->out[i] = fbits(orc_erff_cr(bitsf(c->base + (uint32_t)i)));
}
void orc_erff_range(uint32_t base, uint32_t count, uint32_t *out, int nthreads) {
	struct ef_ctx c = { base, out };
	parallel_rows(ef_rows, &c, (long)count, nthreads);
}

float orc_scale(float x, float s) { return x * s; }

/* ---- soft binary64, restated from StablehloMlx/Kernels/SoftFloat.lean ---------
 * Integer code throughout (independent of the host FPU), with arm64's NaN rules:
 * a NaN operand is returned quieted (first operand first); invalid operations
 * give 0x7FF8000000000000. */
#define FRAC 0xFFFFFFFFFFFFFull
#define HIDDEN 0x10000000000000ull
#define INF64 0x7FF0000000000000ull
#define NAN64 0x7FF8000000000000ull
#define QUIET64 0x8000000000000ull
#define SIGN64 0x8000000000000000ull

static int hibit64(uint64_t x) { return 63 - __builtin_clzll(x); }              /* SoftFloat.lean:40-44 */
static uint64_t srs(uint64_t x, uint32_t n) {                                  /* :47-52 */
	if (n == 0) return x;
	if (n >= 63) return x != 0 ? 1 : 0;
	uint64_t lost = x & ((1ull << n) - 1);
	return (x >> n) | (lost != 0 ? 1 : 0);
}
static uint64_t pack64(uint64_t s, int e, uint64_t m) {                        /* :57-70 */
	if (e < 1) { m = srs(m, (uint32_t)(1 - e)); e = 1; }
	uint64_t rem = m & 0x1FF;
	m >>= 9;
	if (rem > 0x100 || (rem == 0x100 && (m & 1))) m += 1;
	if (m >> 53) { m >>= 1; e += 1; }
	if (e >= 2047) return (s << 63) | INF64;
	uint64_t field = (m >> 52) ? (uint64_t)e : 0;
	return (s << 63) | (field << 52) | (m & FRAC);
}
uint64_t orc_f64_from_f32(float x) {                                           /* :73-85 */
	uint32_t b = fbits(x);
	uint64_t s = b >> 31;
	uint32_t e = (b >> 23) & 0xFF, f = b & 0x7FFFFF;
	if (e == 0xFF) return (s << 63) | INF64 | ((uint64_t)f << 29);
	if (e == 0) {
		if (f == 0) return s << 63;
		uint32_t p = 31 - __builtin_clz(f);
		return (s << 63) | ((uint64_t)(p + 874) << 52) | (((uint64_t)f << (52 - p)) & FRAC);
	}
	return (s << 63) | ((uint64_t)(e + 896) << 52) | ((uint64_t)f << 29);
}
float orc_f64_to_f32(uint64_t d) {                                             /* :95-120 */
	uint32_t s = (uint32_t)(d >> 63);
	int e = (int)((d >> 52) & 0x7FF);
	uint64_t f = d & FRAC;
	if (e == 0x7FF) return bitsf((s << 31) | 0x7F800000u | (f != 0 ? (0x400000u | (uint32_t)(f >> 29)) : 0u));
	if (e == 0 && f == 0) return bitsf(s << 31);
	uint64_t m = f | (e != 0 ? HIDDEN : 0);
	if (e == 0) e = 1;
	int ef = e - 896;
	uint32_t sh = 29;
	if (ef <= 0) { sh = (uint32_t)(30 - ef); ef = 0; }
	if (sh > 63) sh = 63;
	uint64_t q = m >> sh;
	uint64_t rem = m & ((1ull << sh) - 1);
	uint64_t half = 1ull << (sh - 1);
	if (rem > half || (rem == half && (q & 1))) q += 1;
	if (ef == 0) return bitsf((s << 31) | (uint32_t)q);
	if (q >> 24) { q >>= 1; ef += 1; }
	if (ef >= 255) return bitsf((s << 31) | 0x7F800000u);
	return bitsf((s << 31) | ((uint32_t)ef << 23) | (uint32_t)(q & 0x7FFFFF));
}
static void unpack(uint64_t x, int *e, uint64_t *m) {                          /* :124-131 */
	*e = (int)((x >> 52) & 0x7FF);
	*m = x & FRAC;
	if (*e == 0) {
		int h = hibit64(*m);
		*m <<= (52 - h);
		*e = 1 - (52 - h);
	} else {
		*m |= HIDDEN;
	}
}
static int is_nan(uint64_t x) { return (x & 0x7FFFFFFFFFFFFFFFull) > INF64; }
static int is_inf(uint64_t x) { return (x & 0x7FFFFFFFFFFFFFFFull) == INF64; }
static int is_zero(uint64_t x) { return (x & 0x7FFFFFFFFFFFFFFFull) == 0; }

uint64_t orc_f64_add(uint64_t a, uint64_t b) {                                 /* :138-167 */
	if (is_nan(a)) return a | QUIET64;
	if (is_nan(b)) return b | QUIET64;
	if (is_inf(a)) { if (is_inf(b) && a != b) return NAN64; return a; }
	if (is_inf(b)) return b;
	if (is_zero(a)) { if (is_zero(b)) return a & b; return b; }
	if (is_zero(b)) return a;
	uint64_t sa = a >> 63, sb = b >> 63;
	int ae, be;
	uint64_t am, bm;
	unpack(a, &ae, &am);
	unpack(b, &be, &bm);
	am <<= 9; bm <<= 9;
	if (ae < be || (ae == be && am < bm)) {
		int te = ae; ae = be; be = te;
		uint64_t tm = am; am = bm; bm = tm;
		uint64_t ts = sa; sa = sb; sb = ts;
	}
	bm = srs(bm, (uint32_t)(ae - be));
	uint64_t m = (sa == sb) ? am + bm : am - bm;
	if (m == 0) return 0;
	int e = ae;
	int h = hibit64(m);
	if (h > 61) { m = srs(m, 1); e += 1; }
	else { m <<= (61 - h); e -= (61 - h); }
	return pack64(sa, e, m);
}
uint64_t orc_f64_mul(uint64_t a, uint64_t b) {                                 /* :176-197 */
	uint64_t s = (a ^ b) >> 63;
	if (is_nan(a)) return a | QUIET64;
	if (is_nan(b)) return b | QUIET64;
	if (is_inf(a)) { if (is_zero(b)) return NAN64; return (s << 63) | INF64; }
	if (is_inf(b)) { if (is_zero(a)) return NAN64; return (s << 63) | INF64; }
	if (is_zero(a) || is_zero(b)) return s << 63;
	int ae, be;
	uint64_t am, bm;
	unpack(a, &ae, &am);
	unpack(b, &be, &bm);
	unsigned __int128 p = (unsigned __int128)am * bm;   /* leading one at bit 104 or 105 */
	uint64_t lo = (uint64_t)p, hi = (uint64_t)(p >> 64);
	uint64_t m = (hi << 21) | (lo >> 43) | ((lo & 0x7FFFFFFFFFFull) != 0 ? 1 : 0);
	int e = ae + be - 1023;
	if (m >> 62) { m = srs(m, 1); e += 1; }
	return pack64(s, e, m);
}
uint64_t orc_f64_sub(uint64_t a, uint64_t b) {                                 /* :200-204 */
	if (is_nan(a)) return a | QUIET64;
	if (is_nan(b)) return b | QUIET64;
	return orc_f64_add(a, b ^ SIGN64);
}
uint64_t orc_f64_floor(uint64_t a) {                                           /* :207-220 */
	if (is_nan(a)) return a | QUIET64;
	if (is_zero(a)) return a;
	int e = (int)((a >> 52) & 0x7FF);
	if (e >= 1075) return a;
	if (e < 1023) return (a >> 63) ? 0xBFF0000000000000ull : 0;
	uint64_t mask = (1ull << (1075 - e)) - 1;
	if ((a & mask) == 0) return a;
	if ((a >> 63) == 0) return a & ~mask;
	return (a & ~mask) + mask + 1;
}
uint64_t orc_f64_to_i64(uint64_t a) {                                          /* :224-237 */
	if (is_nan(a)) return 0;
	int e = (int)((a >> 52) & 0x7FF);
	uint64_t s = a >> 63;
	if (e < 1023) return 0;
	if (e >= 1086) return s ? SIGN64 : 0x7FFFFFFFFFFFFFFFull;
	uint64_t m = (a & FRAC) | HIDDEN;
	uint64_t q = (e >= 1075) ? (m << (e - 1075)) : (m >> (1075 - e));
	if (s) return (~q) + 1;
	return q;
}
uint64_t orc_f64_div(uint64_t a, uint64_t b) {                                 /* :240-259 */
	uint64_t s = (a ^ b) >> 63;
	if (is_nan(a)) return a | QUIET64;
	if (is_nan(b)) return b | QUIET64;
	if (is_inf(a)) { if (is_inf(b)) return NAN64; return (s << 63) | INF64; }
	if (is_inf(b)) return s << 63;
	if (is_zero(b)) { if (is_zero(a)) return NAN64; return (s << 63) | INF64; }
	if (is_zero(a)) return s << 63;
	int ae, be;
	uint64_t am, bm;
	unpack(a, &ae, &am);
	unpack(b, &be, &bm);
	int e = ae - be + 1023;
	if (am < bm) { am <<= 1; e -= 1; }
	uint64_t r = am, q = 0;
	for (int i = 0; i < 55; i++) {
		q <<= 1;
		if (r >= bm) { r -= bm; q |= 1; }
		r <<= 1;
	}
	uint64_t m = (q << 7) | (r != 0 ? 1 : 0);
	return pack64(s, e, m);
}
float orc_f32_div(float a, float b) {                                          /* :262-264 */
	return orc_f64_to_f32(orc_f64_div(orc_f64_from_f32(a), orc_f64_from_f32(b)));
}
float orc_f32_sqrt(float x) {                                                  /* :267-305 */
	uint32_t b = fbits(x);
	if ((b & 0x7FFFFFFFu) == 0) return x;
	if (b >> 31) return bitsf(0x7FC00000u);
	if (b >= 0x7F800000u) return x;
	int e = (int)(b >> 23);
	uint32_t m = b & 0x7FFFFF;
	if (e == 0) {
		int p = 31 - __builtin_clz(m);
		m <<= (23 - p);
		e = 1 - (23 - p);
	} else {
		m |= 0x800000;
	}
	int k = e - 150;
	uint64_t w = m;
	if (k & 1) { w <<= 1; k -= 1; }
	w <<= 38;
	k -= 38;
	uint64_t r = 0, rem = 0;
	for (int i = 0; i < 32; i++) {
		rem = (rem << 2) | ((w >> 62) & 3);
		w <<= 2;
		uint64_t t = (r << 2) | 1;
		r <<= 1;
		if (rem >= t) { rem -= t; r |= 1; }
	}
	int h = hibit64(r);
	int sh = h - 23;
	uint64_t q = r >> sh;
	uint64_t lost = r & ((1ull << sh) - 1);
	uint64_t half = 1ull << (sh - 1);
	int sticky = rem != 0 || (lost & (half - 1)) != 0;
	if ((lost & half) != 0 && (sticky || (q & 1))) q += 1;
	int ee = (k / 2) + sh + 150;
	if (q >> 24) { q >>= 1; ee += 1; }
	return bitsf(((uint32_t)ee << 23) | (uint32_t)(q & 0x7FFFFF));
}

void orc_f64_ew(int op, const uint64_t *a, const uint64_t *b, uint64_t *y, size_t n) {
	for (size_t i = 0; i < n; i++) {
		uint64_t r = 0;
		switch (op) {
		case 0: r = orc_f64_add(a[i], b[i]); break;
		case 1: r = orc_f64_sub(a[i], b[i]); break;
		case 2: r = orc_f64_mul(a[i], b[i]); break;
		case 3: r = orc_f64_div(a[i], b[i]); break;
		case 4: r = orc_f64_floor(a[i]); break;
		case 5: r = orc_f64_to_i64(a[i]); break;
		default: r = 0;
		}
		y[i] = r;
	}
}
void orc_f64_of_f32_arr(const float *a, uint64_t *y, size_t n) { for (size_t i = 0; i < n; i++) y[i] = orc_f64_from_f32(a[i]); }
void orc_f32_of_f64_arr(const uint64_t *a, float *y, size_t n) { for (size_t i = 0; i < n; i++) y[i] = orc_f64_to_f32(a[i]); }
void orc_f32_div_arr(const float *a, const float *b, float *y, size_t n) { for (size_t i = 0; i < n; i++) y[i] = orc_f32_div(a[i], b[i]); }
void orc_f32_sqrt_arr(const float *a, float *y, size_t n) { for (size_t i = 0; i < n; i++) y[i] = orc_f32_sqrt(a[i]); }
