// Device helpers shared by the spanqr kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace spq {

constexpr int TB = 32;        // Cholesky / triangular-solve tile width (candidates/kchol.py:9 TB = 32)
constexpr int GRAM_TILE = 128;  // Gram output tile (tcgen05 M = N = 128)
constexpr int MAX_R = 512;

// Per-matrix device pointers of one call (filled by k_setup_*).
struct MatPtr {
    const float* X;
    float* Q;
};

// Per-matrix scalars of one pass (written by the Cholesky prologue; read back by tests).
struct PassScal {
    float nrm, shift, tau, s;
};

// Deterministic reciprocal square root: integer-shift seed (0x5f375a86), two Newton steps, one step on the
// fused residual.  Every operation is an explicitly rounded intrinsic so that the compiler cannot contract or
// reorder it: the CPU oracle evaluates the same sequence and gets the same bits.  Within one ulp for normal x > 0.
__device__ __forceinline__ float det_rsqrt(float x) {
    uint32_t i = __float_as_uint(x);
    i = 0x5f375a86u - (i >> 1);
    float y = __uint_as_float(i);
    const float hx = __fmul_rn(0.5f, x);
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        float t = __fmul_rn(hx, y);
        t = __fmul_rn(t, y);
        t = __fsub_rn(1.5f, t);
        y = __fmul_rn(y, t);
    }
    const float e = __fmaf_rn(-x, __fmul_rn(y, y), 1.0f);
    return __fmaf_rn(__fmul_rn(0.5f, y), e, y);
}

// kcholqr.py:29-30 _pow2_scale: 2^-round(log2 max(m, 1e-38)), 1 when m is 0 or NaN, 0 when m is inf.
// log2 is rounded to fp32 first (fp64 log2, then rounded) and round() is half-to-even on that value,
// as torch computes it.
__device__ __forceinline__ float pow2_scale(float m) {
    if (!(m > 0.0f)) return 1.0f;
    if (m < 1e-38f) m = 1e-38f;
    const float l2 = (float)log2((double)m);
    if (isinf(l2)) return 0.0f;
    const float k = rintf(l2);
    return ldexpf(1.0f, -(int)k);
}

// |x| as an unsigned bit pattern: orders non-negative floats, NaN above +inf (so max keeps NaN).
__device__ __forceinline__ uint32_t abs_bits(float x) { return __float_as_uint(x) & 0x7fffffffu; }

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// All threads of a cluster: release this CTA's prior writes, wait for every CTA, acquire theirs.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__host__ __device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// Float-float accumulation (Knuth's two-sum; the square's rounding error from a fused multiply-add): a sum kept as
// hi + lo in two fp32 registers, about 44 significant bits, at the full fp32 rate.  B200 converts fp32 to fp64 at
// about a tenth of its fp64 add rate, so sums of fp32 terms that need more than fp32 accuracy are kept this way and
// converted to fp64 once, at the end.  Every operation is explicitly rounded (no contraction), so the order of the
// terms alone decides the result.
__device__ __forceinline__ void two_sum(float a, float b, float& s, float& e) {
    s = __fadd_rn(a, b);
    const float bb = __fsub_rn(s, a);
    e = __fadd_rn(__fsub_rn(a, __fsub_rn(s, bb)), __fsub_rn(b, bb));
}
// (hi, lo) += x
__device__ __forceinline__ void ff_add(float& hi, float& lo, float x) {
    float s, e;
    two_sum(hi, x, s, e);
    hi = s;
    lo = __fadd_rn(lo, e);
}
// (hi, lo) += x * x, the product split exactly into its rounded value and its error
__device__ __forceinline__ void ff_add_sq(float& hi, float& lo, float x) {
    const float p = __fmul_rn(x, x);
    const float pe = __fmaf_rn(x, x, -p);
    float s, e;
    two_sum(hi, p, s, e);
    hi = s;
    lo = __fadd_rn(lo, __fadd_rn(e, pe));
}
// the float-float value in fp64
__device__ __forceinline__ double ff_value(float hi, float lo) { return __dadd_rn((double)hi, (double)lo); }

// upper-triangular tile index -> (ti, tj) with ti <= tj, row-major over the upper triangle of nt x nt tiles
__device__ __forceinline__ void upper_tile(int t, int nt, int& ti, int& tj) {
    ti = 0;
    while (t >= nt - ti) {
        t -= nt - ti;
        ++ti;
    }
    tj = ti + t;
}

}  // namespace spq
