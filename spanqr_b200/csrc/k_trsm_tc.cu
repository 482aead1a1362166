// Blocked triangular solve Y = (s X + eps Z) L^-T on the tcgen05 tensor cores (candidates/tri.py:378-412, trsm_f).
//
// The reference's 32-column block recurrence Y_j = (A_j - sum_{k<j} Y_k L_jk^T) Li_j^T is evaluated as
//     Y_j = A_j W_jj^T + sum_{k<j} Y_k W_jk^T,   W_jj = Li_j,  W_jk = -Li_j L_jk   (k_trsm_w.cu builds W),
// right-looking: every block's accumulator lives in TMEM from the start (n <= 256: 8 blocks x 32 columns, a large
// hi.hi accumulator and a small hi.lo + lo.hi one, 512 columns), zeroed once, and every product adds to it.  As soon
// as Y_j is known, one product Y_j [W_{j+1, j}; ...; W_{nb-1, j}]^T (N up to 224) updates all later blocks, so the
// chain from one block to the next is only: read the accumulator, write the block, one 32-column product.
// A_{j+1} W_{j+1, j+1}^T is issued while block j is being written, off that chain.
// One CTA = 128 rows of one matrix.  Operands reach shared memory by TMA: 32 x 128 raw tiles of X (or Q) through the
// per-matrix tensor maps (and of the dust Z in the first pass), which the CTA scales, adds and splits into tf32 hi/lo
// operand tiles (K-major, 128B swizzle) in place; the W tiles, already split, by bulk copies of one block column.
// The output block j is written to Q (in place in passes 2 and 3: block j was read before, later blocks are untouched).
#include <cstring>

#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 256;
constexpr int ROWS = 128;
constexpr int BLK = 32;
constexpr int MAXNB = 8;
constexpr int YT = ROWS * 128;                  // 128 rows x 32 fp32 (raw) or tf32 (operand): 16 KB
constexpr int WPART = 4096;                     // 32 x 32 tf32 operand tile
constexpr int OFF_AB = 0;                       // two A buffers [raw x | raw z] -> [hi | lo]: 64 KB
constexpr int OFF_YJ = OFF_AB + 2 * 2 * YT;     // Y_j [hi | lo]: 32 KB
constexpr int OFF_WD = OFF_YJ + 2 * YT;         // two diagonal W tiles [hi | lo]: 16 KB
constexpr int OFF_WT = OFF_WD + 2 * 2 * WPART;  // two trailing W columns [hi tiles | lo tiles]: 2 x 56 KB
constexpr int WTBUF = (MAXNB - 1) * 2 * WPART;
constexpr int OFF_BAR = OFF_WT + 2 * WTBUF;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TCOLS = 512;                 // block c: large at 32 c, small at 256 + 32 c
constexpr int ERR_TIMEOUT = 0x40;
// mbarriers: A tiles landed (x2), diagonal W landed (x2), trailing W landed (x2), accumulator of the next block
// complete, Y_j buffer and trailing W buffer free again, final drain on the error path
enum { B_A = 0, B_WD = 2, B_WT = 4, B_ACC = 6, B_YFREE = 7, B_FIN = 8, NBAR = 9 };
__device__ __forceinline__ uint32_t ring_parity(int c) { return (uint32_t)((c >> 1) & 1); }   // c-th use of a 2-ring
static_assert(TMAP_BOX_COLS == BLK && TMAP_BOX_ROWS == ROWS, "one TMA tile is one 128-row block of 32 columns");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
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

__global__ void __launch_bounds__(NT, 1) k_trsm_tc(PtrArg p, Src src, int K, int n, long long ldq,
                                                   const char* __restrict__ maps, const __grid_constant__ CUtensorMap zmap,
                                                   int has_z, ScaleArg sc, float eps, const char* __restrict__ W_all,
                                                   int* __restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const AB = sm + OFF_AB;
    char* const YJ = sm + OFF_YJ;
    char* const WD = sm + OFF_WD;
    char* const WT = sm + OFF_WT;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 128);

    const int b = blockIdx.y;
    const int row0 = blockIdx.x * ROWS;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    float* Qout = mp.Q;
    const void* amap = maps + ((size_t)b * TMAPS_PER_MATRIX + (src == SRC_X ? 0 : 1)) * 128;
    const int nb = n / BLK;
    const char* Wimg = W_all + (size_t)b * wcol_off(nb, nb);
    float s = 1.0f;
    bool scaled = false;
    if (sc.maxbits) {
        s = pow2_scale(__uint_as_float(sc.maxbits[b]));
        scaled = true;
    } else if (sc.s) {
        s = sc.s[b];
        scaled = true;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i) tc::mbar_init(&bars[i], 1);
        tc::mbar_fence_init();
        tc::tmap_acquire(amap);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tlane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    // every product below adds to its accumulator: start them all at zero
#pragma unroll 1
    for (int c = 0; c < 256; c += 32) tc::tmem_st32_zero(tlane + (uint32_t)((warp >> 2) * 256 + c));
    tc::tmem_wait_st();
    tc::fence_before_sync();

    // copies, issued by thread 0; the counts let the error path wait out whatever is still in flight
    int n_a[2] = {0, 0}, n_wd[2] = {0, 0}, n_wt[2] = {0, 0};
    auto issue_a = [&](int c) {   // raw A_c into A buffer c % 2: x tile, and z tile behind it in the first pass
        uint64_t* bar = &bars[B_A + (c & 1)];
        char* dst = AB + (c & 1) * 2 * YT;
        tc::mbar_expect_tx(bar, has_z ? 2 * YT : YT);
        tc::tma_load_2d(dst, amap, c * BLK, row0, bar);
        if (has_z) tc::tma_load_2d(dst + YT, &zmap, c * BLK, row0, bar);
        ++n_a[c & 1];
    };
    auto issue_wd = [&](int c) {
        uint64_t* bar = &bars[B_WD + (c & 1)];
        tc::mbar_expect_tx(bar, 2 * WPART);
        tc::bulk_g2s(WD + (c & 1) * 2 * WPART, Wimg + wcol_off(nb, c), 2 * WPART, bar);
        ++n_wd[c & 1];
    };
    auto issue_wt = [&](int c) {   // W_{c+1 .. nb-1, c}, c <= nb - 2
        const uint32_t bytes = (uint32_t)(nb - 1 - c) * 2 * WPART;
        uint64_t* bar = &bars[B_WT + (c & 1)];
        tc::mbar_expect_tx(bar, bytes);
        tc::bulk_g2s(WT + (c & 1) * WTBUF, Wimg + wcol_off(nb, c) + 2 * WPART, bytes, bar);
        ++n_wt[c & 1];
    };

    // this thread's slots of an A tile: rows 32 i + am, k-quad aq
    const int aq = tid & 7, am = tid >> 3;
    // A buffer c % 2: raw x (and z) -> s x + eps z -> tf32 hi | lo in place
    auto convert = [&](int c) {
        char* buf = AB + (c & 1) * 2 * YT;
        float4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = 32 * i + am;
            float4 x = *reinterpret_cast<const float4*>(buf + 128 * m + 16 * aq);
            if (scaled) {
                x.x = __fmul_rn(x.x, s); x.y = __fmul_rn(x.y, s); x.z = __fmul_rn(x.z, s); x.w = __fmul_rn(x.w, s);
            }
            if (has_z) {
                const float4 z = *reinterpret_cast<const float4*>(buf + YT + 128 * m + 16 * aq);
                x.x = __fadd_rn(x.x, __fmul_rn(eps, z.x));
                x.y = __fadd_rn(x.y, __fmul_rn(eps, z.y));
                x.z = __fadd_rn(x.z, __fmul_rn(eps, z.z));
                x.w = __fadd_rn(x.w, __fmul_rn(eps, z.w));
            }
            v[i] = x;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) tc::store2_at(buf, buf + YT, tc::swz_off(32 * i + am, aq), v[i]);
        tc::fence_async_smem();
    };
    // D[:, col .. col + N) += A B^T over 32 k (3xTF32: hi.hi large, hi.lo + lo.hi small); A, B: [hi | lo] tile bases
    auto products = [&](uint32_t col, uint32_t ahi_t, uint32_t alo_t, uint32_t bhi_t, uint32_t blo_t, int N) {
        const uint32_t idesc = tc::idesc_tf32(ROWS, N);
#pragma unroll 1
        for (int k = 0; k < 4; ++k) {
            const uint64_t ahi = tc::sdesc_k128(ahi_t + 32 * k), alo = tc::sdesc_k128(alo_t + 32 * k);
            const uint64_t bhi = tc::sdesc_k128(bhi_t + 32 * k), blo = tc::sdesc_k128(blo_t + 32 * k);
            tc::mma_tf32(tmem + col, ahi, bhi, idesc, 1u);
            tc::mma_tf32(tmem + 256 + col, ahi, blo, idesc, 1u);
            tc::mma_tf32(tmem + 256 + col, alo, bhi, idesc, 1u);
        }
    };
    auto diag_products = [&](int c) {   // acc[c] += A_c W_cc^T
        const uint32_t a = tc::smem_u32(AB + (c & 1) * 2 * YT), w = tc::smem_u32(WD + (c & 1) * 2 * WPART);
        products(32 * c, a, a + YT, w, w + WPART, BLK);
    };

    // epilogue mapping: row me (TMEM lane), 16 columns h * 16 .. of the block
    const int me = (warp & 3) * 32 + lane, h = warp >> 2;
    const int rowe = row0 + me;

    if (tid == 0) {
        issue_a(0);
        issue_wd(0);
        if (nb > 1) {
            issue_a(1);
            issue_wd(1);
            issue_wt(0);
        }
        if (nb > 2) issue_wt(1);
    }
    bool ok = __syncthreads_and(tc::mbar_wait(&bars[B_A], 0u) && tc::mbar_wait(&bars[B_WD], 0u));
    if (ok) {
        convert(0);
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
            diag_products(0);
            tc::mma_commit(&bars[B_ACC]);
        }
    }
    for (int j = 0; j < nb && ok; ++j) {
        // the next block's own product, independent of Y_j
        if (j + 1 < nb) {
            const int c = j + 1;
            ok = __syncthreads_and(tc::mbar_wait(&bars[B_A + (c & 1)], ring_parity(c)) &&
                                   tc::mbar_wait(&bars[B_WD + (c & 1)], ring_parity(c)));
            if (!ok) break;
            convert(c);
            tc::fence_before_sync();
            __syncthreads();
            if (tid == 0) {
                tc::fence_after_sync();
                diag_products(c);
            }
        }
        // acc[j] holds A_j W_jj^T + sum_{k<j} Y_k W_jk^T; every product issued before it has completed too
        ok = __syncthreads_and(tc::mbar_wait(&bars[B_ACC], (uint32_t)(j & 1)));
        if (!ok) break;
        tc::fence_after_sync();
        if (tid == 0 && j + 2 < nb) {   // block j's A buffer and diagonal tile are free: block j + 2's go there
            issue_a(j + 2);
            issue_wd(j + 2);
        }
        float big[16], small[16];
        tmem_ld16(tlane + 32 * j + 16 * h, big);
        tmem_ld16(tlane + 256 + 32 * j + 16 * h, small);
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
            bool w = true;
            if (j >= 1) w = tc::mbar_wait(&bars[B_YFREE], (uint32_t)((j - 1) & 1));   // Y_{j-1}'s products are done
            if (w) {
#pragma unroll
                for (int i = 0; i < 4; ++i) tc::store2_at(YJ, YJ + YT, tc::swz_off(me, 4 * h + i), y[i]);
                tc::fence_async_smem();
            }
            w = w && tc::mbar_wait(&bars[B_WT + (j & 1)], ring_parity(j));
            tc::fence_before_sync();
            ok = __syncthreads_and(w);
            if (!ok) break;
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t yj = tc::smem_u32(YJ), wt = tc::smem_u32(WT + (j & 1) * WTBUF);
                const uint32_t lo = (uint32_t)(nb - 1 - j) * WPART;
                products(32 * (j + 1), yj, yj + YT, wt, wt + lo, BLK);   // block j + 1 first: its epilogue waits on it
                tc::mma_commit(&bars[B_ACC]);
                if (j + 2 < nb) products(32 * (j + 2), yj, yj + YT, wt + WPART, wt + lo + WPART, BLK * (nb - 2 - j));
                tc::mma_commit(&bars[B_YFREE]);
                // the trailing buffer of block j - 1 was freed by the wait above: column j + 1 goes there
                if (j >= 1 && j + 1 <= nb - 2) issue_wt(j + 1);
            }
        }
    }
    if (!ok && tid == 0) {
        atomicOr(status, ERR_TIMEOUT);
        // let issued copies and products finish before this CTA's shared memory and TMEM are released
        for (int i = 0; i < 2; ++i) {
            if (n_a[i]) tc::mbar_wait(&bars[B_A + i], (uint32_t)((n_a[i] - 1) & 1));
            if (n_wd[i]) tc::mbar_wait(&bars[B_WD + i], (uint32_t)((n_wd[i] - 1) & 1));
            if (n_wt[i]) tc::mbar_wait(&bars[B_WT + i], (uint32_t)((n_wt[i] - 1) & 1));
        }
        tc::mma_commit(&bars[B_FIN]);
        tc::mbar_wait(&bars[B_FIN], 0u);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

size_t trsm_w_bytes(int n) { return wcol_off(n / BLK, n / BLK); }

cudaError_t launch_trsm_tc(PtrArg p, Src src, int K, int n, long long ldq, int B, const char* maps, const float* Z,
                           ScaleArg sc, float eps, const char* W, int* status, cudaStream_t st) {
    if (n > MAXNB * BLK || n % BLK) return cudaErrorInvalidValue;
    alignas(64) CUtensorMap zmap;
    memset(&zmap, 0, sizeof(zmap));
    if (Z) {
        cudaError_t e = encode_rows(&zmap, Z, K, n, n, TMAP_BOX_COLS, TMAP_BOX_ROWS);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaFuncSetAttribute(k_trsm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k_trsm_tc<<<dim3((K + ROWS - 1) / ROWS, B), NT, SMEM_BYTES, st>>>(p, src, K, n, ldq, maps, zmap, Z ? 1 : 0, sc, eps,
                                                                    W, status);
    return cudaGetLastError();
}

}  // namespace spq
