// Block Gram-Schmidt for r > 512 (candidates/kbig.py:66-95, BCGS2 over 256-column blocks): the pieces around the
// Gram (k_gram_tc in band mode) and the update (k_ns_ws in projection mode) -- the scaled copy of a block of X into
// Q, and the operand image of -T from the band's split partials.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

// Q[:, 0 .. w) = s X[:, 0 .. w) (kbig.py: W = X[:, j:j+b] * s, s = _pow2_scale(max |X|), a power of 2)
__global__ void __launch_bounds__(256) k_scale_copy(const float* __restrict__ X, long long ldx, float* __restrict__ Q,
                                                    long long ldq, int K, int w, const uint32_t* __restrict__ maxbits) {
    const float s = pow2_scale(__uint_as_float(*maxbits));
    const int w4 = w / 4;
    const long long n4 = (long long)K * w4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / w4;
        const int col = (int)(i - row * w4) * 4;
        float4 v = __ldg(reinterpret_cast<const float4*>(X + row * ldx + col));
        v.x = __fmul_rn(v.x, s);
        v.y = __fmul_rn(v.y, s);
        v.z = __fmul_rn(v.z, s);
        v.w = __fmul_rn(v.w, s);
        *reinterpret_cast<float4*>(Q + row * ldq + col) = v;
    }
}

// -T (T = P^T W, P = the first j columns, W = the next 256) as the projection's B operand: for each chunk of 32
// contraction indices (columns of P), rows c = 0..255 (columns of W) x 32 k, K-major with the 128-byte swizzle, the
// tf32 hi part then the lo part.  One thread: column c of W, contraction quad kq; the band's split partials are summed
// in split order in float-float and rounded once (kbig.py's fp32 P^T W; the sum order is fixed by (K, j)).
__global__ void __launch_bounds__(256) k_band_image(const float* __restrict__ P, GramPlan gp, int j,
                                                    char* __restrict__ img_all) {
    const int b = blockIdx.y;
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (j / 4) * BLOCK_W) return;
    const int c = e % BLOCK_W, kq = e / BLOCK_W, kc = kq / 8, q = kq % 8;
    const int ti = 4 * kq / GRAM_TILE, u = 4 * kq % GRAM_TILE;
    const int tj = c / GRAM_TILE, v = c % GRAM_TILE;   // tile column within the band
    const int tile = ti * (gp.nt - gp.b0) + tj;
    float hi[4] = {0.f, 0.f, 0.f, 0.f}, lo[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < gp.S; ++sp) {
        const float* pt = P + ((size_t)(b * gp.S + sp) * gp.tiles + tile) * GRAM_TILE * GRAM_TILE + (size_t)u * GRAM_TILE + v;
#pragma unroll
        for (int i = 0; i < 4; ++i) ff_add(hi[i], lo[i], __ldg(pt + i * GRAM_TILE));
    }
    const float4 t = make_float4(-__fadd_rn(hi[0], lo[0]), -__fadd_rn(hi[1], lo[1]), -__fadd_rn(hi[2], lo[2]),
                                 -__fadd_rn(hi[3], lo[3]));
    char* part = img_all + (size_t)b * band_img_bytes(j) + (size_t)kc * 2 * BLOCK_W * 128;
    tc::store2_at(part, part + (size_t)BLOCK_W * 128, tc::swz_off(c, q), t);
}

cudaError_t launch_scale_copy(const float* X, long long ldx, float* Q, long long ldq, int K, int w,
                              const uint32_t* maxbits, cudaStream_t st) {
    if (w % 4 || ldx % 4 || ldq % 4) return cudaErrorInvalidValue;
    const long long n4 = (long long)K * (w / 4);
    long long blocks = (n4 + 256 * 4 - 1) / (256 * 4);
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    k_scale_copy<<<(int)blocks, 256, 0, st>>>(X, ldx, Q, ldq, K, w, maxbits);
    return cudaGetLastError();
}

cudaError_t launch_band_image(const float* P, const GramPlan& gp, int j, char* img, cudaStream_t st) {
    if (j < BLOCK_W || j % BLOCK_W || gp.b0 * GRAM_TILE != j) return cudaErrorInvalidValue;
    k_band_image<<<dim3(cdiv(j / 4 * BLOCK_W, 256), 1), 256, 0, st>>>(P, gp, j, img);
    return cudaGetLastError();
}

}  // namespace spq
