// Blocked triangular solve Y = (s X + eps Z) L^-T on the tcgen05 tensor cores (candidates/tri.py:378-412, trsm_f).
//
// One CTA = 128 rows of one matrix, n <= 256 columns in 32-column blocks j (the reference's blocking):
//     Y_j = (A_j - sum_{k<j} Y_k L[j, k]^T) Li_j^T,   Li_j = inverse of the 32 x 32 diagonal tile of L.
// The finished blocks of the current 128-column panel stay in shared memory as tf32 hi/lo MMA operands (K-major,
// 128B swizzle).  Per block: the off-diagonal sum over the panel's earlier blocks is one run of tcgen05.mma
// M128 N32 K8 products (hi.hi into one TMEM accumulator, hi.lo + lo.hi into a second); the second panel of a
// 256-column matrix first takes the whole first panel's contribution as one M128 N128 K128 product into its own pair
// of TMEM accumulators.  Then each row (two threads per row, 16 output columns each) forms v = A_j - contributions and
// multiplies by Li_j^T on the CUDA cores (32 x 16 fused multiply-adds), writes Y_j to the output (in place when the
// input is the output: block j is read before it is written and later blocks are not touched), and splits it into the
// shared operand tiles for the next blocks.  The 3xTF32 products are fp32-accurate; the reference's solve uses tf32x3.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 256;
constexpr int ROWS = 128;
constexpr int BLK = 32;
constexpr int YT = ROWS * 128;            // one 128-row x 32-k operand tile (16 KB)
constexpr int LB = BLK * 128;             // one 32-row x 32-k operand tile (4 KB)
constexpr int OFF_YP = 0;                 // [4 blocks][hi, lo] Y panel tiles: 128 KB
constexpr int OFF_LS = 8 * YT;            // L staging: in-panel [3 k-chunks][hi, lo] x 4 KB, or panel [2][hi, lo] x 16 KB
constexpr int OFF_LI = OFF_LS + 4 * YT;   // Li_j transposed, 32 x 32 floats
constexpr int OFF_BAR = OFF_LI + 4096;
constexpr int SMEM_BYTES = OFF_BAR + 1024 + 1024;
constexpr uint32_t TCOLS = 512;           // panel large [0,128) small [128,256); block large [256,288) small [288,320)
constexpr int ERR_TIMEOUT = 0x40;
}  // namespace

__global__ void __launch_bounds__(NT, 1) k_trsm_tc(PtrArg p, Src src, int K, int n, long long ldx, long long ldq,
                                                   const float* __restrict__ Z, ScaleArg sc, float eps,
                                                   const float* __restrict__ L_all, const float* __restrict__ Li_all,
                                                   int* __restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const YP = sm + OFF_YP;
    char* const LS = sm + OFF_LS;
    float* const LIt = reinterpret_cast<float*>(sm + OFF_LI);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);   // [0] block sum done, [1,2] panel chunk buffer free,
                                                                  // [3] panel product done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 64);

    const int b = blockIdx.y;
    const int row0 = blockIdx.x * ROWS;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    const float* Xin = (src == SRC_X) ? mp.X : mp.Q;
    const long long ldin = (src == SRC_X) ? ldx : ldq;
    float* Qout = mp.Q;
    const float* L = L_all + (size_t)b * n * n;
    const float* Li = Li_all + (size_t)b * n * BLK;
    float s = 1.0f;
    bool scaled = false;
    if (sc.maxbits) {
        s = pow2_scale(__uint_as_float(sc.maxbits[b]));
        scaled = true;
    } else if (sc.s) {
        s = sc.s[b];
        scaled = true;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = warp >> 2;                       // this thread's half of a block's 32 columns
    const int m = (warp & 3) * 32 + lane;          // this thread's row in the block (its TMEM lane)
    const int row = row0 + m;
    const bool rin = row < K;
    const int nb = n / BLK;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) tc::mbar_init(&bars[i], 1);
        tc::mbar_fence_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tlane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t id_blk = tc::idesc_tf32(ROWS, BLK), id_pan = tc::idesc_tf32(ROWS, 128);
    bool ok = true;
    int blk_commits = 0;

    for (int j = 0; j < nb && ok; ++j) {
        const int pl = j >> 2, jl = j & 3;

        if (jl == 0 && pl == 1) {
            // panel product C = Y[:, 0:128] L[128:256, 0:128]^T, L streamed in 32-column chunks (two buffers)
            for (int kc = 0; kc < 4 && ok; ++kc) {
                const int bb = kc & 1;
                bool w = true;
                if (kc >= 2) w = tc::mbar_wait(&bars[1 + bb], 0u);
                ok = __syncthreads_and(w);
                if (!ok) break;
                char* t = LS + bb * 2 * YT;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 8 * ((warp & 3) * 4 + i) + (lane & 7), q = (warp >> 2) * 4 + (lane >> 3);
                    const float4 v = __ldg(reinterpret_cast<const float4*>(L + (size_t)(128 + r) * n + kc * BLK + 4 * q));
                    tc::store2_at(t, t + YT, tc::swz_off(r, q), v);
                }
                tc::fence_async_smem();
                __syncthreads();
                if (threadIdx.x == 0) {
                    tc::fence_after_sync();
                    const uint32_t a = tc::smem_u32(YP + kc * 2 * YT), bt = tc::smem_u32(t);
#pragma unroll 1
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t acc_in = (kc > 0 || k > 0) ? 1u : 0u;
                        const uint64_t ahi = tc::sdesc_k128(a + 32 * k), alo = tc::sdesc_k128(a + YT + 32 * k);
                        const uint64_t bhi = tc::sdesc_k128(bt + 32 * k), blo = tc::sdesc_k128(bt + YT + 32 * k);
                        tc::mma_tf32(tmem, ahi, bhi, id_pan, acc_in);
                        tc::mma_tf32(tmem + 128, ahi, blo, id_pan, acc_in);
                        tc::mma_tf32(tmem + 128, alo, bhi, id_pan, 1u);
                    }
                    tc::mma_commit(&bars[1 + bb]);
                    if (kc == 3) tc::mma_commit(&bars[3]);
                }
            }
            if (!ok) break;
            ok = __syncthreads_and(tc::mbar_wait(&bars[3], 0u));   // the panel-0 tiles may now be overwritten
            if (!ok) break;
        }

        // stage the in-panel operand L[j, pl*128 + 32 kc ...] (kc < jl) and Li_j (transposed)
        for (int kc = 0; kc < jl; ++kc) {
            const int r = threadIdx.x >> 3, q = threadIdx.x & 7;
            const float4 v = __ldg(reinterpret_cast<const float4*>(L + (size_t)(j * BLK + r) * n + pl * 128 + kc * BLK + 4 * q));
            char* t = LS + kc * 2 * LB;
            tc::store2_at(t, t + LB, tc::swz_off(r, q), v);
        }
#pragma unroll
        for (int e = threadIdx.x; e < BLK * BLK; e += NT) {
            const int cp = e >> 5, c = e & 31;                 // Li[j*32 + cp][c] -> LIt[c][cp]
            LIt[c * BLK + cp] = __ldg(Li + (size_t)(j * BLK + cp) * BLK + c);
        }
        tc::fence_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        if (jl > 0 && threadIdx.x == 0) {
            tc::fence_after_sync();
            const uint32_t ypb = tc::smem_u32(YP), lsb = tc::smem_u32(LS);
            for (int kc = 0; kc < jl; ++kc) {
#pragma unroll 1
                for (int k = 0; k < 4; ++k) {
                    const uint32_t acc_in = (kc > 0 || k > 0) ? 1u : 0u;
                    const uint32_t a = ypb + kc * 2 * YT, bt = lsb + kc * 2 * LB;
                    const uint64_t ahi = tc::sdesc_k128(a + 32 * k), alo = tc::sdesc_k128(a + YT + 32 * k);
                    const uint64_t bhi = tc::sdesc_k128(bt + 32 * k), blo = tc::sdesc_k128(bt + LB + 32 * k);
                    tc::mma_tf32(tmem + 256, ahi, bhi, id_blk, acc_in);
                    tc::mma_tf32(tmem + 288, ahi, blo, id_blk, acc_in);
                    tc::mma_tf32(tmem + 288, alo, bhi, id_blk, 1u);
                }
            }
            tc::mma_commit(&bars[0]);
        }

        // this thread's row of A_j (32 columns), while the MMAs run
        float v[32];
        {
            const float* xr = Xin + (long long)row * ldin + j * BLK;
            const float* zr = Z ? Z + (long long)row * n + j * BLK : nullptr;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                float4 x = rin ? *reinterpret_cast<const float4*>(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                if (scaled) {
                    x.x = __fmul_rn(x.x, s); x.y = __fmul_rn(x.y, s); x.z = __fmul_rn(x.z, s); x.w = __fmul_rn(x.w, s);
                }
                if (zr && rin) {
                    const float4 z = __ldg(reinterpret_cast<const float4*>(zr + i));
                    x.x = __fadd_rn(x.x, __fmul_rn(eps, z.x));
                    x.y = __fadd_rn(x.y, __fmul_rn(eps, z.y));
                    x.z = __fadd_rn(x.z, __fmul_rn(eps, z.z));
                    x.w = __fadd_rn(x.w, __fmul_rn(eps, z.w));
                }
                v[i] = x.x; v[i + 1] = x.y; v[i + 2] = x.z; v[i + 3] = x.w;
            }
        }
        if (jl > 0) {
            ok = __syncthreads_and(tc::mbar_wait(&bars[0], (uint32_t)(blk_commits & 1)));
            ++blk_commits;
            if (!ok) break;
        }
        tc::fence_after_sync();
        if (pl == 1) {                                  // first panel's contribution
            float t0[32], t1[32];
            tc::tmem_ld32(tlane + 32 * jl, t0);
            tc::tmem_ld32(tlane + 128 + 32 * jl, t1);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __fsub_rn(v[i], __fadd_rn(t0[i], t1[i]));
        }
        if (jl > 0) {                                   // this panel's earlier blocks
            float t0[32], t1[32];
            tc::tmem_ld32(tlane + 256, t0);
            tc::tmem_ld32(tlane + 288, t1);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __fsub_rn(v[i], __fadd_rn(t0[i], t1[i]));
        }
        // y[c'] = sum_c v[c] Li_j[c'][c] for this thread's 16 columns c' = 16 h + i
        float y[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < BLK; ++c) {
            const float4* lrow = reinterpret_cast<const float4*>(LIt + c * BLK + 16 * h);
#pragma unroll
            for (int i4 = 0; i4 < 4; ++i4) {
                const float4 l = lrow[i4];
                y[4 * i4] = __fmaf_rn(v[c], l.x, y[4 * i4]);
                y[4 * i4 + 1] = __fmaf_rn(v[c], l.y, y[4 * i4 + 1]);
                y[4 * i4 + 2] = __fmaf_rn(v[c], l.z, y[4 * i4 + 2]);
                y[4 * i4 + 3] = __fmaf_rn(v[c], l.w, y[4 * i4 + 3]);
            }
        }
        // every thread has read this block's TMEM and the operand staging: the next block may reuse them
        tc::fence_before_sync();
        __syncthreads();
        if (rin) {
            float* qr = Qout + (long long)row * ldq + j * BLK + 16 * h;
#pragma unroll
            for (int i4 = 0; i4 < 4; ++i4)
                *reinterpret_cast<float4*>(qr + 4 * i4) = make_float4(y[4 * i4], y[4 * i4 + 1], y[4 * i4 + 2], y[4 * i4 + 3]);
        }
        if (j + 1 < nb) {
            char* t = YP + jl * 2 * YT;
#pragma unroll
            for (int i4 = 0; i4 < 4; ++i4)
                tc::store2_at(t, t + YT, tc::swz_off(m, 4 * h + i4),
                              make_float4(y[4 * i4], y[4 * i4 + 1], y[4 * i4 + 2], y[4 * i4 + 3]));
        }
    }
    if (!ok && threadIdx.x == 0) atomicOr(status, ERR_TIMEOUT);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

cudaError_t launch_trsm_tc(PtrArg p, Src src, int K, int n, long long ldx, long long ldq, int B, const float* Z,
                           ScaleArg sc, float eps, const float* L, const float* Li, int* status, cudaStream_t st) {
    if (n > 256 || n % BLK) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_trsm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k_trsm_tc<<<dim3((K + ROWS - 1) / ROWS, B), NT, SMEM_BYTES, st>>>(p, src, K, n, ldx, ldq, Z, sc, eps, L, Li, status);
    return cudaGetLastError();
}

}  // namespace spq
