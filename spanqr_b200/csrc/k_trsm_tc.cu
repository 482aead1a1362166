// Blocked triangular solve Y = (s X + eps Z) L^-T on the tcgen05 tensor cores (candidates/tri.py:378-412, trsm_f).
//
// The reference's 32-column block recurrence Y_j = (A_j - sum_{k<j} Y_k L_jk^T) Li_j^T is evaluated as
//     Y_j = A_j W_jj^T + sum_{k<j} Y_k W_jk^T,   W_jj = Li_j,  W_jk = -Li_j L_jk   (k_trsm_w.cu builds W),
// so every block is one chain of tensor-core products and nothing but a copy sits between two blocks.
// One CTA = 128 rows of one matrix, n <= 256 columns.  The finished blocks of the current 128-column panel stay in
// shared memory as tf32 hi/lo operands (K-major, 128B swizzle); per block j the CTA splits A_j into the same form,
// has W_jk (already split, in the shared-memory layout) copied in by cp.async one block ahead, and one thread issues
// tcgen05.mma M128 N32 K8 products (hi.hi into one TMEM accumulator, hi.lo + lo.hi into a second).  The second panel
// of a 256-column matrix starts from one M128 N128 K128 product of the first panel with W[4..7, 0..3] in the same
// accumulators.  Each block's result is written to the output (in place when the input is the output: block j is read
// before it is written, later blocks are not touched) and split into the operand tiles of the next blocks.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 256;
constexpr int ROWS = 128;
constexpr int BLK = 32;
constexpr int YT = ROWS * 128;            // 128-row x 32-k operand tile (16 KB)
constexpr int WPART = 4096;               // 32-row x 32-k operand tile (4 KB)
constexpr int OFF_YP = 0;                 // [4 blocks][hi, lo] panel tiles: 128 KB
constexpr int OFF_A = 8 * YT;             // A_j [hi, lo]: 32 KB
constexpr int OFF_W = OFF_A + 2 * YT;     // two W buffers of 32 KB
constexpr int WBUF = 2 * YT;
constexpr int OFF_BAR = OFF_W + 2 * WBUF;
constexpr int SMEM_BYTES = OFF_BAR + 128 + 1024;
constexpr uint32_t TCOLS = 256;           // large [0,128), small [128,256): one 32-column slot per block of a panel
constexpr int ERR_TIMEOUT = 0x40;
}  // namespace

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(NT, 1) k_trsm_tc(PtrArg p, Src src, int K, int n, long long ldx, long long ldq,
                                                   const float* __restrict__ Z, ScaleArg sc, float eps,
                                                   const char* __restrict__ W_all, int* __restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const YP = sm + OFF_YP;
    char* const AB = sm + OFF_A;
    char* const WS = sm + OFF_W;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);   // [0] block done, [1,2] panel buffer free, [3] panel done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 64);

    const int b = blockIdx.y;
    const int row0 = blockIdx.x * ROWS;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    const float* Xin = (src == SRC_X) ? mp.X : mp.Q;
    const long long ldin = (src == SRC_X) ? ldx : ldq;
    float* Qout = mp.Q;
    const int nb = n / BLK, ntile = nb * (nb + 1) / 2;
    const char* Wimg = W_all + (size_t)b * ntile * 2 * WPART;
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

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) tc::mbar_init(&bars[i], 1);
        tc::mbar_fence_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t id_blk = tc::idesc_tf32(ROWS, BLK), id_pan = tc::idesc_tf32(ROWS, 128);

    // in-panel W tiles of block j (k = first block of its panel .. j) into buffer bf, 16 bytes per copy
    auto issue_w = [&](int j, int bf) {
        const int k0 = (j >> 2) * 4;
        const int bytes = (j - k0 + 1) * 2 * WPART;
        const char* src0 = Wimg + (size_t)(j * (j + 1) / 2 + k0) * 2 * WPART;   // tiles (j, k0 .. j) are consecutive
        for (int o = threadIdx.x * 16; o < bytes; o += NT * 16) tc::cp_async16(WS + bf * WBUF + o, src0 + o);
        tc::cp_async_commit();
    };

    // this thread's A-tile slots: rows m = 8 * ((warp & 3) * 4 + i) + (lane & 7), k-quad q
    const int aq = (warp >> 2) * 4 + (lane >> 3);
    float4 ra[4];
    auto load_a = [&](int j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = 8 * ((warp & 3) * 4 + i) + (lane & 7);
            const int row = row0 + m, col = j * BLK + 4 * aq;
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (row < K) {
                x = *reinterpret_cast<const float4*>(Xin + (long long)row * ldin + col);
                if (scaled) {
                    x.x = __fmul_rn(x.x, s); x.y = __fmul_rn(x.y, s); x.z = __fmul_rn(x.z, s); x.w = __fmul_rn(x.w, s);
                }
                if (Z) {
                    const float4 z = __ldg(reinterpret_cast<const float4*>(Z + (long long)row * n + col));
                    x.x = __fadd_rn(x.x, __fmul_rn(eps, z.x));
                    x.y = __fadd_rn(x.y, __fmul_rn(eps, z.y));
                    x.z = __fadd_rn(x.z, __fmul_rn(eps, z.z));
                    x.w = __fadd_rn(x.w, __fmul_rn(eps, z.w));
                }
            }
            ra[i] = x;
        }
    };

    // epilogue mapping: row me (TMEM lane), 16 columns h * 16 .. of the block
    const int me = (warp & 3) * 32 + lane, h = warp >> 2;
    const int rowe = row0 + me;
    const uint32_t tlane = tmem + ((uint32_t)((warp & 3) * 32) << 16);

    bool ok = true;
    issue_w(0, 0);
    load_a(0);
    for (int j = 0; j < nb && ok; ++j) {
        const int pl = j >> 2, jl = j & 3;
        if (jl == 0 && pl == 1) {
            // first panel's contribution to the second: sum_{kc<4} Y_kc W[4..7, kc]^T, W streamed by column block
            for (int kc = 0; kc < 4 && ok; ++kc) {
                const int bb = kc & 1;
                bool w = true;
                if (kc >= 2) w = tc::mbar_wait(&bars[1 + bb], 0u);
                ok = __syncthreads_and(w);
                if (!ok) break;
                for (int jj = 0; jj < 4; ++jj) {
                    const int jr = 4 + jj;
                    const char* t = Wimg + (size_t)(jr * (jr + 1) / 2 + kc) * 2 * WPART;
                    for (int part = 0; part < 2; ++part)
                        for (int o = threadIdx.x * 16; o < WPART; o += NT * 16)
                            tc::cp_async16(WS + bb * WBUF + part * YT + jj * WPART + o, t + part * WPART + o);
                }
                tc::cp_async_commit();
                tc::cp_async_wait<0>();
                tc::fence_async_smem();
                __syncthreads();
                if (threadIdx.x == 0) {
                    tc::fence_after_sync();
                    const uint32_t a = tc::smem_u32(YP + kc * 2 * YT), bt = tc::smem_u32(WS + bb * WBUF);
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
            ok = __syncthreads_and(tc::mbar_wait(&bars[3], 0u));   // panel-0 tiles and both W buffers are free
            if (!ok) break;
            issue_w(j, j & 1);
        }

        // A_j -> operand tiles (the previous block's products have completed), prefetch A_{j+1}
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = 8 * ((warp & 3) * 4 + i) + (lane & 7);
            tc::store2_at(AB, AB + YT, tc::swz_off(m, aq), ra[i]);
        }
        if (j + 1 < nb) load_a(j + 1);
        tc::cp_async_wait<0>();                          // this block's W tiles have landed
        if (j + 1 < nb && ((j + 1) & 3) != 0) issue_w(j + 1, (j + 1) & 1);
        tc::fence_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
            tc::fence_after_sync();
            const uint32_t dbig = tmem + 32 * jl, dsmall = tmem + 128 + 32 * jl;
            const uint32_t wb = tc::smem_u32(WS + (j & 1) * WBUF);
            const uint32_t start = (pl == 1) ? 1u : 0u;    // the second panel adds to the first panel's product
            // A_j W_jj^T: W tile jl of the buffer
            {
                const uint32_t a = tc::smem_u32(AB), bt = wb + jl * 2 * WPART;
#pragma unroll 1
                for (int k = 0; k < 4; ++k) {
                    const uint32_t acc_in = (k > 0) ? 1u : start;
                    const uint64_t ahi = tc::sdesc_k128(a + 32 * k), alo = tc::sdesc_k128(a + YT + 32 * k);
                    const uint64_t bhi = tc::sdesc_k128(bt + 32 * k), blo = tc::sdesc_k128(bt + WPART + 32 * k);
                    tc::mma_tf32(dbig, ahi, bhi, id_blk, acc_in);
                    tc::mma_tf32(dsmall, ahi, blo, id_blk, acc_in);
                    tc::mma_tf32(dsmall, alo, bhi, id_blk, 1u);
                }
            }
            // Y_k W_jk^T for the panel's earlier blocks k
            for (int kc = 0; kc < jl; ++kc) {
                const uint32_t a = tc::smem_u32(YP + kc * 2 * YT), bt = wb + kc * 2 * WPART;
#pragma unroll 1
                for (int k = 0; k < 4; ++k) {
                    const uint64_t ahi = tc::sdesc_k128(a + 32 * k), alo = tc::sdesc_k128(a + YT + 32 * k);
                    const uint64_t bhi = tc::sdesc_k128(bt + 32 * k), blo = tc::sdesc_k128(bt + WPART + 32 * k);
                    tc::mma_tf32(dbig, ahi, bhi, id_blk, 1u);
                    tc::mma_tf32(dsmall, ahi, blo, id_blk, 1u);
                    tc::mma_tf32(dsmall, alo, bhi, id_blk, 1u);
                }
            }
            tc::mma_commit(&bars[0]);
        }
        ok = __syncthreads_and(tc::mbar_wait(&bars[0], (uint32_t)(j & 1)));
        if (!ok) break;
        tc::fence_after_sync();
        float big[16], small[16];
        tmem_ld16(tlane + 32 * jl + 16 * h, big);
        tmem_ld16(tlane + 128 + 32 * jl + 16 * h, small);
        tc::tmem_wait_ld();
        float4 y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            y[i] = make_float4(__fadd_rn(big[4 * i], small[4 * i]), __fadd_rn(big[4 * i + 1], small[4 * i + 1]),
                               __fadd_rn(big[4 * i + 2], small[4 * i + 2]), __fadd_rn(big[4 * i + 3], small[4 * i + 3]));
        if (rowe < K) {
            float* qr = Qout + (long long)rowe * ldq + j * BLK + 16 * h;
#pragma unroll
            for (int i = 0; i < 4; ++i) *reinterpret_cast<float4*>(qr + 4 * i) = y[i];
        }
        if (j + 1 < nb) {
            char* t = YP + jl * 2 * YT;
#pragma unroll
            for (int i = 0; i < 4; ++i) tc::store2_at(t, t + YT, tc::swz_off(me, 4 * h + i), y[i]);
        }
        tc::fence_before_sync();
    }
    if (!ok && threadIdx.x == 0) atomicOr(status, ERR_TIMEOUT);
    tc::cp_async_wait<0>();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

size_t trsm_w_bytes(int n) {
    const int nb = n / BLK;
    return (size_t)nb * (nb + 1) / 2 * 2 * WPART;
}

cudaError_t launch_trsm_tc(PtrArg p, Src src, int K, int n, long long ldx, long long ldq, int B, const float* Z,
                           ScaleArg sc, float eps, const char* W, int* status, cudaStream_t st) {
    if (n > 256 || n % BLK) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_trsm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k_trsm_tc<<<dim3((K + ROWS - 1) / ROWS, B), NT, SMEM_BYTES, st>>>(p, src, K, n, ldx, ldq, Z, sc, eps, W, status);
    return cudaGetLastError();
}

}  // namespace spq
