// Blocked triangular solve Y = (s X + eps Z) L^-T on the tcgen05 tensor cores (candidates/tri.py:378-412, trsm_f).
//
// The reference's 32-column block recurrence Y_j = (A_j - sum_{k<j} Y_k L_jk^T) Li_j^T is evaluated as
//     Y_j = A_j W_jj^T + sum_{k<j} Y_k W_jk^T,   W_jj = Li_j,  W_jk = -Li_j L_jk   (k_trsm_w.cu builds W),
// right-looking: every block's accumulator lives in TMEM from the start (n <= 256: 8 blocks x 32 columns, a large
// hi.hi accumulator and a small hi.lo + lo.hi one, 512 columns), zeroed once, and every product adds to it.
// One CTA = 128 rows of one matrix, in four warp roles:
//   warps 0-3  epilogue: TMEM lanes 0-127 = the CTA's rows; block j's accumulators -> Y_j -> output rows and the
//              tf32 hi/lo operand of the update;
//   warps 4-7  convert: raw 32 x 128 tiles of X (or Q, and the dust Z in the first pass) -> s x + eps z -> tf32 hi/lo
//              operand tiles (K-major, 128B swizzle), in place;
//   warp 8     one thread issues every product, in a fixed order, so the result does not depend on timing;
//   warp 9     one thread issues every copy: row tiles through the per-matrix tensor maps, W tiles by bulk copy (a
//              copy can hold its issuing thread for a microsecond, which must not delay the products).
// Block c's row tile, its operand and later Y_c share one slot of a ring of three (raw -> hi | lo -> Y_c hi | lo), so
// the update by Y_j never waits for a buffer the next block needs.  Product order, fixed in code:
//   diag(0); [ACC]; then for j = 0 .. nb-2:  diag(j+1) (before Y_j exists: it overlaps block j's epilogue);
//   T(j) = Y_j W_{j+1.., j}^T into every later block (one product, N = 32 (nb - 1 - j)); [ACC: block j+1 complete];
//   [FREE of slot j % 3].
// A product costs the same whatever its N, so one stacked update per step is cheaper than splitting off block j+1.
// The output block j is written to Q (in place in passes 2 and 3: block j was read before, later blocks are untouched).
// One launch solves one panel of at most 8 blocks, j0 .. j0 + nbp - 1, of a matrix of NB = n / 32 blocks (W indexed in
// the whole image); a second panel starts its accumulators from `init`, the first panel's contribution
// sum_{k < j0} Y_k W_jk^T computed by k_ns_ws in its product mode.
#include <cstring>

#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 320;                         // 4 epilogue warps, 4 convert warps, a product warp, a copy warp
constexpr int ROWS = 128;
constexpr int BLK = 32;
constexpr int MAXNB = 8;
constexpr int YT = ROWS * 128;                  // 128 rows x 32 fp32 (raw) or tf32 (operand): 16 KB
constexpr int WPART = 4096;                     // 32 x 32 tf32 operand tile
constexpr int NSLOT = 3;                        // row-block slots [raw x | raw z] -> [hi | lo] -> [Y hi | Y lo]
constexpr int SLOT = 2 * YT;
constexpr int OFF_AB = 0;
constexpr int OFF_WD = OFF_AB + NSLOT * SLOT;   // two diagonal W tiles [hi | lo]: 16 KB
constexpr int OFF_WT = OFF_WD + 2 * 2 * WPART;  // two trailing W columns [hi tiles | lo tiles]: 2 x 56 KB
constexpr int WTBUF = (MAXNB - 1) * 2 * WPART;
constexpr int OFF_BAR = OFF_WT + 2 * WTBUF;
constexpr int BAR_BYTES = 512;
constexpr int SMEM_BYTES = OFF_BAR + BAR_BYTES + 1024;
constexpr uint32_t TCOLS = 512;                 // block c: large at 32 c, small at 256 + 32 c
constexpr int ERR_TIMEOUT = 0x40;
// mbarriers: row tile landed (per slot), diagonal W landed (x2), trailing W landed (x2), operand converted (per slot,
// 128 arrivals), Y_j stored (128 arrivals), accumulator of the next block complete, slot released (per slot: the update
// by its Y and everything issued before it done), error drain.  A parity wait is only meaningful for the phase
// in progress or the one just completed: every waiter below steps through its barrier's phases in order from phase 0,
// and no barrier can run two phases ahead of a waiter, because its next phase needs something that waiter has not yet
// released (the copy thread's one wait on ACC phase 0 comes before it issues the diagonal tile that ACC phase 2
// needs).
enum { B_A = 0, B_WD = 3, B_WT = 5, B_CONV = 7, B_Y = 10, B_ACC = 11, B_FREE = 12, B_FIN = 15, NBAR = 16 };
__device__ __forceinline__ uint32_t par2(int c) { return (uint32_t)((c >> 1) & 1); }   // c-th use of a 2-ring
__device__ __forceinline__ uint32_t par3(int c) { return (uint32_t)((c / 3) & 1); }    // c-th use of a 3-ring
static_assert(TMAP_BOX_COLS == BLK && TMAP_BOX_ROWS == ROWS, "one TMA tile is one 128-row block of 32 columns");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(NBAR * 8 + 16 <= BAR_BYTES, "barrier area");
}  // namespace

__global__ void __launch_bounds__(NT, 1) k_trsm_tc(PtrArg p, Src src, int K, int n, long long ldq, int j0, int nbp,
                                                   const float* __restrict__ init,
                                                   const char* __restrict__ maps, const __grid_constant__ CUtensorMap zmap,
                                                   int has_z, ScaleArg sc, float eps, const char* __restrict__ W_all,
                                                   int* __restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const AB = sm + OFF_AB;
    char* const WD = sm + OFF_WD;
    char* const WT = sm + OFF_WT;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + NBAR * 8);
    volatile int* err = reinterpret_cast<volatile int*>(sm + OFF_BAR + NBAR * 8 + 4);

    const int b = blockIdx.y;
    const int row0 = blockIdx.x * ROWS;
    const int NB = n / BLK;   // blocks of the matrix (W image)
    const int nb = nbp;       // blocks of this panel, j0 .. j0 + nb - 1; local index c <-> block j0 + c
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i)
            tc::mbar_init(&bars[i], ((i >= B_CONV && i < B_CONV + NSLOT) || i == B_Y) ? 128 : 1);
        tc::mbar_fence_init();
        *err = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------- epilogue warps: row me of the CTA ----------------
        const uint32_t tlane = tmem + ((uint32_t)(warp * 32) << 16);
        // every product adds to its accumulator: start them at zero, or the large ones at `init` (this row)
#pragma unroll 1
        for (int c = 0; c < (int)TCOLS; c += 32) {
            if (init && c < 32 * nb) {
                const int row = row0 + warp * 32 + lane;
                float v[32];
                const float* ir = init + ((size_t)b * K + (row < K ? row : 0)) * 256 + c;
                if (row < K) {
                    tc::ld_row32(ir, v, true);   // workspace rows: 1 KB apart, 256-byte aligned base
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.f;
                }
                tc::tmem_st32(tlane + (uint32_t)c, v);
            } else {
                tc::tmem_st32_zero(tlane + (uint32_t)c);
            }
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        tc::bar_sync(2, 128 + 32);   // with the issue warp: accumulators zeroed before the first product
        const int me = warp * 32 + lane, rowe = row0 + me;
        float* qrow = (p.tab ? p.tab[b] : p.one).Q + (long long)rowe * ldq;
        const bool w8 = tc::al32(qrow);   // 32-byte stores where the row allows them
        // exits are decided per warp (__all_sync): tcgen05.ld needs the whole warp
        for (int j = 0; j < nb; ++j) {
            if (!__all_sync(0xffffffffu, !*err && tc::mbar_wait(&bars[B_ACC], (uint32_t)(j & 1)))) {   // acc[j] done
                *err = 1;
                break;
            }
            tc::fence_after_sync();
            float big[32], small[32];
            tc::tmem_ld32(tlane + 32 * j, big);
            tc::tmem_ld32(tlane + 256 + 32 * j, small);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) big[i] = __fadd_rn(big[i], small[i]);
            if (j + 1 < nb) {   // Y_j into block j's slot: its operand was last read by diag(j), complete with acc[j]
                char* slot = AB + (j % NSLOT) * SLOT;
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    tc::store2_at(slot, slot + YT, tc::swz_off(me, q),
                                  make_float4(big[4 * q], big[4 * q + 1], big[4 * q + 2], big[4 * q + 3]));
                tc::fence_async_smem();
                tc::mbar_arrive(&bars[B_Y]);
            }
            if (rowe < K) tc::st_row32(qrow + 32 * (j0 + j), big, w8);
        }
    } else if (warp < 8) {
        // ---------------- convert warps: raw A_c -> s x + eps z -> tf32 hi | lo, in place ----------------
        float s = 1.0f;
        bool scaled = false;
        if (sc.maxbits) {
            s = pow2_scale(__uint_as_float(sc.maxbits[b]));
            scaled = true;
        } else if (sc.s) {
            s = sc.s[b];
            scaled = true;
        }
        const int t = tid - 128, aq = t & 7, am = t >> 3;   // rows 16 i + am, k-quad aq
        // exits are decided by the whole group (bar_and): it meets again at a named barrier
        for (int c = 0; c < nb; ++c) {
            if (!tc::bar_and(1, 128, !*err && tc::mbar_wait(&bars[B_A + c % NSLOT], par3(c)))) {
                *err = 1;
                break;
            }
            char* buf = AB + (c % NSLOT) * SLOT;
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int m = 16 * i + am;
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
            tc::bar_sync(1, 128);   // every convert thread has read the raw tile before it is overwritten
#pragma unroll
            for (int i = 0; i < 8; ++i) tc::store2_at(buf, buf + YT, tc::swz_off(16 * i + am, aq), v[i]);
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[B_CONV + c % NSLOT]);
        }
    } else if (warp == 8) {
        // ---------------- product warp ----------------
        tc::bar_sync(2, 128 + 32);
        if (lane == 0) {
            // D[:, col .. col + N) += A B^T over 32 k (3xTF32: hi.hi large, hi.lo + lo.hi small)
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
            auto diag = [&](int c) -> bool {   // acc[c] += A_c W_cc^T
                if (*err || !tc::mbar_wait(&bars[B_CONV + c % NSLOT], par3(c)) || !tc::mbar_wait(&bars[B_WD + (c & 1)], par2(c)))
                    return false;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_u32(AB + (c % NSLOT) * SLOT), w = tc::smem_u32(WD + (c & 1) * 2 * WPART);
                products(32 * c, a, a + YT, w, w + WPART, BLK);
                return true;
            };
            bool ok = diag(0);
            if (ok) tc::mma_commit(&bars[B_ACC]);
            for (int j = 0; ok && j + 1 < nb; ++j) {
                ok = diag(j + 1) && !*err && tc::mbar_wait(&bars[B_Y], (uint32_t)(j & 1)) &&
                     tc::mbar_wait(&bars[B_WT + (j & 1)], par2(j));
                if (!ok) break;
                tc::fence_after_sync();
                const int t = nb - 1 - j;   // trailing tiles of column j in this panel: blocks j + 1 .. nb - 1
                const uint32_t yj = tc::smem_u32(AB + (j % NSLOT) * SLOT), wt = tc::smem_u32(WT + (j & 1) * WTBUF);
                // blocks j + 1 .. nb - 1 in one product (block j + 1 is then complete)
                products(32 * (j + 1), yj, yj + YT, wt, wt + (uint32_t)t * WPART, BLK * t);
                tc::mma_commit(&bars[B_ACC]);
                tc::mma_commit(&bars[B_FREE + j % NSLOT]);
            }
            if (!ok) {
                *err = 1;
                tc::mma_commit(&bars[B_FIN]);   // let issued products finish before TMEM is released
                tc::mbar_wait(&bars[B_FIN], 0u);
            }
        }
    } else {
        // ---------------- copy warp ----------------
        if (lane == 0) {
            const void* amap = maps + ((size_t)b * TMAPS_PER_MATRIX + (src == SRC_X ? TMAP_X : TMAP_Q)) * 128;
            const char* Wimg = W_all + (size_t)b * wcol_off(NB, NB);
            tc::tmap_acquire(amap);
            int n_a[NSLOT] = {0, 0, 0}, n_wd[2] = {0, 0}, n_wt[2] = {0, 0};
            auto issue_a = [&](int c) {   // raw A_c into slot c % 3: x tile, and z tile behind it in the first pass
                uint64_t* bar = &bars[B_A + c % NSLOT];
                char* dst = AB + (c % NSLOT) * SLOT;
                tc::mbar_expect_tx(bar, has_z ? 2 * YT : YT);
                tc::tma_load_2d(dst, amap, (j0 + c) * BLK, row0, bar);
                if (has_z) tc::tma_load_2d(dst + YT, &zmap, (j0 + c) * BLK, row0, bar);
                ++n_a[c % NSLOT];
            };
            auto issue_wd = [&](int c) {
                uint64_t* bar = &bars[B_WD + (c & 1)];
                tc::mbar_expect_tx(bar, 2 * WPART);
                tc::bulk_g2s(WD + (c & 1) * 2 * WPART, Wimg + wcol_off(NB, j0 + c), 2 * WPART, bar);
                ++n_wd[c & 1];
            };
            auto issue_wt = [&](int c) {   // W_{c+1 .. nb-1, c} of the panel (local indices), c <= nb - 2
                const int g = j0 + c, t = nb - 1 - c;   // the column's trailing tiles in the panel: the first t
                uint64_t* bar = &bars[B_WT + (c & 1)];
                const char* hi = Wimg + wcol_off(NB, g) + 2 * WPART;
                tc::mbar_expect_tx(bar, (uint32_t)t * 2 * WPART);
                if (NB - 1 - g == t) {   // the panel runs to the last block: hi and lo tiles adjacent, one copy
                    tc::bulk_g2s(WT + (c & 1) * WTBUF, hi, (uint32_t)t * 2 * WPART, bar);
                } else {
                    tc::bulk_g2s(WT + (c & 1) * WTBUF, hi, (uint32_t)t * WPART, bar);
                    tc::bulk_g2s(WT + (c & 1) * WTBUF + t * WPART, hi + (size_t)(NB - 1 - g) * WPART, (uint32_t)t * WPART,
                                 bar);
                }
                ++n_wt[c & 1];
            };
            bool ok = true;
            for (int c = 0; c < nb && c < NSLOT; ++c) issue_a(c);
            for (int c = 0; c < nb && c < 2; ++c) issue_wd(c);
            for (int c = 0; c + 1 < nb && c < 2; ++c) issue_wt(c);
            if (nb > 2) {   // diag(0) done: its tile's buffer takes W_22
                ok = !*err && tc::mbar_wait(&bars[B_ACC], 0u);
                if (ok) issue_wd(2);
            }
            for (int j = 0; ok && j + 2 < nb; ++j) {
                // slot j % 3 released: T(j) and diag(j + 1) (issued before it) are complete
                ok = !*err && tc::mbar_wait(&bars[B_FREE + j % NSLOT], par3(j));
                if (!ok) break;
                if (j + 3 < nb) {
                    issue_a(j + 3);    // into slot j % 3 (Y_j consumed)
                    issue_wd(j + 3);   // into W_{j+1,j+1}'s buffer (diag(j + 1) done)
                }
                if (j + 2 <= nb - 2) issue_wt(j + 2);   // into column j's buffer
            }
            if (!ok) {
                *err = 1;
                // let issued copies finish before this CTA's shared memory is released
                for (int i = 0; i < NSLOT; ++i)
                    if (n_a[i]) tc::mbar_wait(&bars[B_A + i], (uint32_t)((n_a[i] - 1) & 1));
                for (int i = 0; i < 2; ++i) {
                    if (n_wd[i]) tc::mbar_wait(&bars[B_WD + i], (uint32_t)((n_wd[i] - 1) & 1));
                    if (n_wt[i]) tc::mbar_wait(&bars[B_WT + i], (uint32_t)((n_wt[i] - 1) & 1));
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0 && *err) atomicOr(status, ERR_TIMEOUT);
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

size_t trsm_w_bytes(int n) { return wcol_off(n / BLK, n / BLK); }

cudaError_t launch_trsm_tc(PtrArg p, Src src, int K, int n, long long ldq, int B, int j0, int nbp, const float* init,
                           const char* maps, const float* Z, long long ldz, ScaleArg sc, float eps, const char* W,
                           int* status, cudaStream_t st) {
    if (n > 512 || n % BLK || nbp < 1 || nbp > MAXNB || j0 < 0 || (j0 + nbp) * BLK > n) return cudaErrorInvalidValue;
    alignas(64) CUtensorMap zmap;
    memset(&zmap, 0, sizeof(zmap));
    if (Z) {
        cudaError_t e = encode_rows(&zmap, Z, K, n, ldz, TMAP_BOX_COLS, TMAP_BOX_ROWS);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaFuncSetAttribute(k_trsm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k_trsm_tc<<<dim3((K + ROWS - 1) / ROWS, B), NT, SMEM_BYTES, st>>>(p, src, K, n, ldq, j0, nbp, init, maps, zmap,
                                                                    Z ? 1 : 0, sc, eps, W, status);
    return cudaGetLastError();
}

}  // namespace spq
