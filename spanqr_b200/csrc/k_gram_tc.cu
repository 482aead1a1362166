// Gram G = A^T A (A = s Y, Y [K, n] fp32 row-major) on the 5th-generation tensor cores, split-TF32 (3xTF32).
//
// One CTA = one 128 x 128 tile (ti <= tj) of the upper triangle of G over one 512-row split of Y.  Per 32-row chunk
// the 256 threads load the two 32 x 128 column panels with coalesced 16-byte loads (warp w: rows 4w .. 4w+3, lane l:
// columns 4l .. 4l+3), split every value into tf32 parts and store them into MN-major shared tiles (128-byte swizzle
// on a 32-byte base, the MN-major layout tcgen05 takes for tf32) --
// the Gram contracts over the rows of Y, so Y's own row-major layout is the MN-major operand layout and no transpose
// is needed; one thread then issues, per k-step of 8 rows, tcgen05.mma M128 N128 K8 products:
//   plain mode    (x = hi + lo, 22 of 24 bits): hi.hi | hi.lo + lo.hi                                   (3 MMAs)
//   accurate mode (x = hi + mid + lo exactly):  hi.hi | hi.mid + mid.hi + hi.lo + mid.mid + lo.hi      (6 MMAs)
// hi.hi goes to one TMEM accumulator and the small products to a second one, so the small terms never round
// against the large partial sum.  After every group of rows the large-term accumulator is drained into fp64 registers
// while the next group accumulates in the other TMEM buffer; the small-term accumulator (about 2^-11 of the total) stays in
// TMEM for the whole split and is drained once at the end.  The split's fp64 sum is rounded to fp32 and written as a
// partial.  k_gram_reduce
// (k_gram.cu) sums the partials in split order.  Which mode runs where: the orth
// sequence uses the drained mode for its last polish Gram (the reference's compensated gram_split, kcholqr.py:20) and
// the plain mode for the Grams of r > 256 (k_gram_ws covers r <= 256) and, with a band plan (tiles ti < b0 <= tj), for
// T = P^T W of block Gram-Schmidt (r > 512); the accurate mode serves the component entry point spanqr_gram_f32, the
// counterpart of the reference's compensated gram_f / gram_split (tri.py:285-375).
// Determinism: the split size (512 rows) and every order depend only on (K, n), never on the batch or the GPU.
// Compensation: the reference (candidates/tri.py:255-375) Kahan-sums fp32 32-row dots inside a split and adds the
// splits in fp64; here each group of rows (32 in the accurate mode, 128 in the drained mode) sums its products in the
// tensor core's fp32 and the groups are added in fp64.
// The tensor core's fp32 accumulation rounds toward zero, so a sum of same-sign products drifts low by about half
// an ulp per accumulation (measured: -19 ulps of sum |y_i y_j| after 128 rows on the diagonal, under 2.3 ulps off the
// diagonal of an orthonormal Y).  The diagonal -- every column's sum of squares, the entries that set the final
// orthogonality -- is therefore computed on the CUDA cores from the same scaled values (squares split exactly into
// value and error, float-float sums in a fixed order) by the diagonal-tile CTAs and written over the tensor-core
// diagonal.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int TILE = 128;
constexpr int CHUNK = 32;
constexpr int OPND = 16384;     // one 128 x 32 tf32 operand tile
constexpr int ERR_TIMEOUT = 0x10;
// per buffer: A parts then B parts (PARTS = 2: hi, lo; PARTS = 3: hi, mid, lo)
template <int PARTS> constexpr int buf_bytes() { return 2 * PARTS * OPND; }
template <int PARTS> constexpr int smem_bytes() { return 2 * buf_bytes<PARTS>() + 1024 /*barriers*/ + 1024 /*alignment*/; }
constexpr uint32_t TMEM_COLS = 512;  // large-term accumulators at 0 and 128 (two groups), small-term at 256
}  // namespace

GramPlan gram_tc_plan(int K, int n) {
    GramPlan g;
    g.nt = (n + TILE - 1) / TILE;
    g.tiles = g.nt * (g.nt + 1) / 2;
    g.KS = GRAM_TC_SPLIT;
    g.S = (K + g.KS - 1) / g.KS;
    g.b0 = 0;
    return g;
}

// the band of block Gram-Schmidt: 512-row splits, doubled (up to 2048 rows) while the grid still has four CTAs per SM,
// so that tall matrices write fewer partials; a function of (K, j) only
GramPlan gram_band_plan(int K, int j) {
    GramPlan g;
    g.b0 = j / TILE;
    g.nt = g.b0 + BLOCK_W / TILE;
    g.tiles = g.b0 * (g.nt - g.b0);
    g.KS = GRAM_TC_SPLIT;
    while (g.KS < 4 * GRAM_TC_SPLIT && (long long)g.tiles * ((K + 2 * g.KS - 1) / (2 * g.KS)) >= 4 * 148) g.KS *= 2;
    g.S = (K + g.KS - 1) / g.KS;
    return g;
}

constexpr int NT = 256;         // 8 warps: 4 TMEM lane quadrants x 2 column halves of the 128 x 128 tile

template <int PARTS>
__global__ void __launch_bounds__(NT, 1) k_gram_tc(PtrArg p, Src src, int K, int n, long long ld, GramPlan gp,
                                                    ScaleArg sc, float* __restrict__ P, int* __restrict__ status) {
    // chunks per fp64 drain of the large-term accumulator: every 32 rows in the accurate mode (the truncated fp32
    // accumulation of same-sign products then spans 4 MMAs), every 128 rows in the plain mode
    constexpr int GROUP = (PARTS == 3) ? 1 : 4;
    constexpr int BUF = buf_bytes<PARTS>();
    constexpr int BOFF = PARTS * OPND;   // B parts follow the A parts
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const buf0 = reinterpret_cast<char*>(sm);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 2 * BUF);   // [0,1] operand buffer free, [2,3] accumulator full
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + 2 * BUF + 64);

    const int tile = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
    int ti, tj;
    gram_tile_of(gp, tile, ti, tj);
    const bool diag = ti == tj;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    const float* __restrict__ Y = (src == SRC_X) ? mp.X : mp.Q;
    float s = 1.0f;
    bool scaled = false;
    if (sc.maxbits) {
        s = pow2_scale(__uint_as_float(sc.maxbits[b]));
        scaled = true;
    } else if (sc.s) {
        s = sc.s[b];
        scaled = true;
    }
    const int k0 = sp * gp.KS;
    const int k1 = min(k0 + gp.KS, K);
    const int nchunks = (k1 - k0 + CHUNK - 1) / CHUNK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TMEM_COLS);
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) tc::mbar_init(&bars[i], 1);
        tc::mbar_fence_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    // this thread's slots of a 32 x 128 panel: rows 4 * warp + i (i = 0..3), columns 4 * lane .. 4 * lane + 3; a
    // warp's 16-byte stores for one row fill one 128-byte row of each of the 4 MN-atoms: no bank conflict
    const int colA = ti * TILE + 4 * lane, colB = tj * TILE + 4 * lane;
    const bool inA = colA < n, inB = !diag && colB < n;   // n is a multiple of 32, so 4 columns are in or out together
    uint32_t soff[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) soff[i] = tc::swz_mn_off(4 * warp + i, 4 * lane);

    auto load = [&](int c, float4 (&ra)[4], float4 (&rb)[4]) {
        const int row0 = k0 + c * CHUNK + 4 * warp;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = row0 + i;
            const float* yr = Y + (long long)row * ld;
            float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
            if (row < k1) {
                if (inA) va = __ldg(reinterpret_cast<const float4*>(yr + colA));
                if (inB) vb = __ldg(reinterpret_cast<const float4*>(yr + colB));
            }
            if (scaled) {
                va.x = __fmul_rn(va.x, s); va.y = __fmul_rn(va.y, s); va.z = __fmul_rn(va.z, s); va.w = __fmul_rn(va.w, s);
                vb.x = __fmul_rn(vb.x, s); vb.y = __fmul_rn(vb.y, s); vb.z = __fmul_rn(vb.z, s); vb.w = __fmul_rn(vb.w, s);
            }
            ra[i] = va;
            rb[i] = vb;
        }
    };
    float sqh[4] = {0.f, 0.f, 0.f, 0.f}, sql[4] = {0.f, 0.f, 0.f, 0.f};   // diagonal tiles: squares of colA .. + 3
    auto stage = [&](int bi, const float4 (&ra)[4], const float4 (&rb)[4]) {
        char* base = buf0 + bi * BUF;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (diag) {
                ff_add_sq(sqh[0], sql[0], ra[i].x);
                ff_add_sq(sqh[1], sql[1], ra[i].y);
                ff_add_sq(sqh[2], sql[2], ra[i].z);
                ff_add_sq(sqh[3], sql[3], ra[i].w);
            }
            if constexpr (PARTS == 2) tc::store2_at(base, base + OPND, soff[i], ra[i]);
            else tc::store3_at(base, base + OPND, base + 2 * OPND, soff[i], ra[i]);
            if (!diag) {
                if constexpr (PARTS == 2) tc::store2_at(base + BOFF, base + BOFF + OPND, soff[i], rb[i]);
                else tc::store3_at(base + BOFF, base + BOFF + OPND, base + BOFF + 2 * OPND, soff[i], rb[i]);
            }
        }
    };

    double acc[64];   // rows (warp & 3) * 32 + lane, columns (warp >> 2) * 64 .. + 64
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.0;
    const uint32_t idesc = tc::idesc_tf32_mn(TILE, TILE);
    const uint32_t tq = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * 64);
    const uint32_t tsmall = tmem + 2 * TILE;

    // add 64 accumulator columns at TMEM address t (this thread's lane) into acc
    auto add_cols = [&](uint32_t t) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float v[32];
            tc::tmem_ld32(t + 32 * h, v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[32 * h + i] = __dadd_rn(acc[32 * h + i], (double)v[i]);
        }
    };
    auto drain = [&](int g, bool last) -> bool {
        const int gb = g & 1;
        bool ok = tc::mbar_wait(&bars[2 + gb], (uint32_t)((g >> 1) & 1));
        ok = __syncthreads_and(ok);
        if (!ok) return false;
        tc::fence_after_sync();
        add_cols(tq + gb * TILE);
        if (last) add_cols(tq + 2 * TILE);   // this thread's lanes and columns of the small-term accumulator
        tc::fence_before_sync();
        return true;
    };

    auto chunk = [&](int c, float4 (&ra)[4], float4 (&rb)[4]) -> bool {
        const int bi = c & 1;
        bool ok = true;
        if (c >= 2) ok = tc::mbar_wait(&bars[bi], (uint32_t)(((c - 2) >> 1) & 1));
        ok = __syncthreads_and(ok);
        if (!ok) return false;
        stage(bi, ra, rb);
        tc::fence_async_smem();
        if (c + 2 < nchunks) load(c + 2, ra, rb);
        __syncthreads();
        const int g = c / GROUP;
        if (threadIdx.x == 0) {
            tc::fence_after_sync();
            const uint32_t abase = tc::smem_u32(buf0 + bi * BUF);
            const uint32_t bbase = diag ? abase : abase + BOFF;
            const uint32_t dbig = tmem + (uint32_t)((g & 1) * TILE), dsmall = tsmall;
#pragma unroll 1
            for (int k = 0; k < CHUNK / 8; ++k) {
                const uint32_t acc_in = (c % GROUP != 0 || k > 0) ? 1u : 0u;          // large: per group
                const uint32_t acc_small = (c != 0 || k > 0) ? 1u : 0u;              // small: whole split
                // k-step k = rows 8k .. 8k+7 of the chunk = k-atoms 2k, 2k+1 (2048 bytes apart); MN-atoms 512 apart
                const uint64_t ahi = tc::sdesc_mn128b32(abase + 4096 * k, 512, 2048);
                const uint64_t alo = tc::sdesc_mn128b32(abase + (PARTS - 1) * OPND + 4096 * k, 512, 2048);
                const uint64_t bhi = tc::sdesc_mn128b32(bbase + 4096 * k, 512, 2048);
                const uint64_t blo = tc::sdesc_mn128b32(bbase + (PARTS - 1) * OPND + 4096 * k, 512, 2048);
                tc::mma_tf32(dbig, ahi, bhi, idesc, acc_in);
                if constexpr (PARTS == 2) {
                    tc::mma_tf32(dsmall, ahi, blo, idesc, acc_small);
                    tc::mma_tf32(dsmall, alo, bhi, idesc, 1u);
                } else {
                    const uint64_t amid = tc::sdesc_mn128b32(abase + OPND + 4096 * k, 512, 2048);
                    const uint64_t bmid = tc::sdesc_mn128b32(bbase + OPND + 4096 * k, 512, 2048);
                    tc::mma_tf32(dsmall, ahi, bmid, idesc, acc_small);
                    tc::mma_tf32(dsmall, amid, bhi, idesc, 1u);
                    tc::mma_tf32(dsmall, ahi, blo, idesc, 1u);
                    tc::mma_tf32(dsmall, amid, bmid, idesc, 1u);
                    tc::mma_tf32(dsmall, alo, bhi, idesc, 1u);
                }
            }
            tc::mma_commit(&bars[bi]);
            if (c % GROUP == GROUP - 1 || c == nchunks - 1) tc::mma_commit(&bars[2 + (g & 1)]);
        }
        if (c % GROUP == 0 && g >= 1) return drain(g - 1, false);
        return true;
    };

    float4 ra0[4], rb0[4], ra1[4], rb1[4];
    load(0, ra0, rb0);
    if (nchunks > 1) load(1, ra1, rb1);
    bool ok = true;
    for (int c = 0; c < nchunks && ok; c += 2) {
        ok = chunk(c, ra0, rb0);
        if (ok && c + 1 < nchunks) ok = chunk(c + 1, ra1, rb1);
    }
    if (ok) ok = drain((nchunks - 1) / GROUP, true);

    if (ok) {
        const int row = (warp & 3) * 32 + lane;
        float* ptile = P + ((size_t)(b * gp.S + sp) * gp.tiles + tile) * TILE * TILE;
        float* out = ptile + (size_t)row * TILE + (warp >> 2) * 64;
        // partial rows: 512 bytes apart, 256-byte aligned base
#pragma unroll
        for (int h = 0; h < 64; h += 32) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __double2float_rn(acc[h + i]);
            tc::st_row32(out + h, v, true);
        }
        if (diag) {
            // fixed-order sum of the 8 warps' partial sums of squares of each column (warp order 0..7); overwrite the
            // diagonal of the partial tile
            double* dsum = reinterpret_cast<double*>(buf0);   // operand buffers are free: every MMA has completed
#pragma unroll
            for (int j = 0; j < 4; ++j) dsum[warp * TILE + 4 * lane + j] = ff_value(sqh[j], sql[j]);
            __syncthreads();
            if (threadIdx.x < TILE) {
                const int m = threadIdx.x;
                double t = dsum[m];
                for (int w = 1; w < NT / 32; ++w) t = __dadd_rn(t, dsum[w * TILE + m]);
                ptile[(size_t)m * TILE + m] = __double2float_rn(t);
            }
        }
    } else if (threadIdx.x == 0) {
        atomicOr(status, ERR_TIMEOUT);
        // a wait ran out: give the MMAs already issued a bounded chance to finish before TMEM is released
        const int last = nchunks - 1;
        tc::mbar_wait(&bars[2 + ((last / GROUP) & 1)], (uint32_t)(((last / GROUP) >> 1) & 1));
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

// Plain mode (the reference's SGEMM Grams: passes 2 and 3 and the first polish step): two CTAs per SM instead of one,
// so each CTA's load latency and barriers are hidden by the other's work.  Per CTA one operand buffer (hi, lo of both
// panels: 64 KB), the whole 512-row split accumulated in TMEM (hi.hi and hi.lo + lo.hi in separate 128-column
// accumulators, 256 columns), no fp64 drains; the exact fp64 diagonal as in the accurate mode.  Same tile/split plan
// and partial layout as k_gram_tc.
constexpr int PLAIN_NT = 256;
constexpr int PLAIN_BUF = 4 * OPND;
constexpr int PLAIN_SMEM = PLAIN_BUF + 1024 + 1024;

__global__ void __launch_bounds__(PLAIN_NT, 2) k_gram_tc_plain(PtrArg p, Src src, int K, int n, long long ld, GramPlan gp,
                                                                ScaleArg sc, float* __restrict__ P, int* __restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const buf = reinterpret_cast<char*>(sm);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + PLAIN_BUF);   // [0] operand buffer free
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + PLAIN_BUF + 64);
    const int tile = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
    int ti, tj;
    gram_tile_of(gp, tile, ti, tj);
    const bool diag = ti == tj;
    const MatPtr mp = p.tab ? p.tab[b] : p.one;
    const float* __restrict__ Y = (src == SRC_X) ? mp.X : mp.Q;
    float s = 1.0f;
    bool scaled = false;
    if (sc.maxbits) {
        s = pow2_scale(__uint_as_float(sc.maxbits[b]));
        scaled = true;
    } else if (sc.s) {
        s = sc.s[b];
        scaled = true;
    }
    const int k0 = sp * gp.KS;
    const int k1 = min(k0 + gp.KS, K);
    const int nchunks = (k1 - k0 + CHUNK - 1) / CHUNK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t TC = 256;
    if (warp == 0) tc::tmem_alloc(tmem_slot, TC);
    if (threadIdx.x == 0) {
        tc::mbar_init(&bars[0], 1);
        tc::mbar_fence_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = tc::idesc_tf32_mn(TILE, TILE);
    const int colA = ti * TILE + 4 * lane, colB = tj * TILE + 4 * lane;
    const bool inA = colA < n, inB = !diag && colB < n;
    uint32_t soff[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) soff[i] = tc::swz_mn_off(4 * warp + i, 4 * lane);
    float4 ra[4], rb[4];
    auto load = [&](int c) {
        const int row0 = k0 + c * CHUNK + 4 * warp;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = row0 + i;
            const float* yr = Y + (long long)row * ld;
            float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
            if (row < k1) {
                if (inA) va = __ldg(reinterpret_cast<const float4*>(yr + colA));
                if (inB) vb = __ldg(reinterpret_cast<const float4*>(yr + colB));
            }
            if (scaled) {
                va.x = __fmul_rn(va.x, s); va.y = __fmul_rn(va.y, s); va.z = __fmul_rn(va.z, s); va.w = __fmul_rn(va.w, s);
                vb.x = __fmul_rn(vb.x, s); vb.y = __fmul_rn(vb.y, s); vb.z = __fmul_rn(vb.z, s); vb.w = __fmul_rn(vb.w, s);
            }
            ra[i] = va;
            rb[i] = vb;
        }
    };
    float sqh[4] = {0.f, 0.f, 0.f, 0.f}, sql[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    load(0);
    for (int c = 0; c < nchunks; ++c) {
        if (c >= 1) ok = tc::mbar_wait(&bars[0], (uint32_t)((c - 1) & 1));   // the previous chunk's MMAs are done
        ok = __syncthreads_and(ok);
        if (!ok) break;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (diag) {
                ff_add_sq(sqh[0], sql[0], ra[i].x);
                ff_add_sq(sqh[1], sql[1], ra[i].y);
                ff_add_sq(sqh[2], sql[2], ra[i].z);
                ff_add_sq(sqh[3], sql[3], ra[i].w);
            }
            tc::store2_at(buf, buf + OPND, soff[i], ra[i]);
            if (!diag) tc::store2_at(buf + 2 * OPND, buf + 3 * OPND, soff[i], rb[i]);
        }
        tc::fence_async_smem();
        if (c + 1 < nchunks) load(c + 1);
        __syncthreads();
        if (threadIdx.x == 0) {
            tc::fence_after_sync();
            const uint32_t abase = tc::smem_u32(buf);
            const uint32_t bbase = diag ? abase : abase + 2 * OPND;
#pragma unroll 1
            for (int k = 0; k < CHUNK / 8; ++k) {
                const uint32_t acc_in = (c > 0 || k > 0) ? 1u : 0u;
                const uint64_t ahi = tc::sdesc_mn128b32(abase + 4096 * k, 512, 2048);
                const uint64_t alo = tc::sdesc_mn128b32(abase + OPND + 4096 * k, 512, 2048);
                const uint64_t bhi = tc::sdesc_mn128b32(bbase + 4096 * k, 512, 2048);
                const uint64_t blo = tc::sdesc_mn128b32(bbase + OPND + 4096 * k, 512, 2048);
                tc::mma_tf32(tmem, ahi, bhi, idesc, acc_in);
                tc::mma_tf32(tmem + TILE, ahi, blo, idesc, acc_in);
                tc::mma_tf32(tmem + TILE, alo, bhi, idesc, 1u);
            }
            tc::mma_commit(&bars[0]);
        }
    }
    if (ok) ok = __syncthreads_and(tc::mbar_wait(&bars[0], (uint32_t)((nchunks - 1) & 1)));
    if (ok) {
        tc::fence_after_sync();
        const int row = (warp & 3) * 32 + lane;
        float* ptile = P + ((size_t)(b * gp.S + sp) * gp.tiles + tile) * TILE * TILE;
        const uint32_t tq = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * 64);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float v[32], w[32];
            tc::tmem_ld32(tq + 32 * hh, v);
            tc::tmem_ld32(tq + TILE + 32 * hh, w);
            tc::tmem_wait_ld();
            float* out = ptile + (size_t)row * TILE + (warp >> 2) * 64 + 32 * hh;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(out + i) = make_float4(__fadd_rn(v[i], w[i]), __fadd_rn(v[i + 1], w[i + 1]),
                                                                  __fadd_rn(v[i + 2], w[i + 2]), __fadd_rn(v[i + 3], w[i + 3]));
        }
        if (diag) {
            double* dsum = reinterpret_cast<double*>(buf);   // operand buffer is free: every MMA has completed
#pragma unroll
            for (int j = 0; j < 4; ++j) dsum[warp * TILE + 4 * lane + j] = ff_value(sqh[j], sql[j]);
            __syncthreads();
            if (threadIdx.x < TILE) {
                const int m = threadIdx.x;
                double t = dsum[m];
                for (int w2 = 1; w2 < PLAIN_NT / 32; ++w2) t = __dadd_rn(t, dsum[w2 * TILE + m]);
                ptile[(size_t)m * TILE + m] = __double2float_rn(t);
            }
        }
    } else if (threadIdx.x == 0) {
        atomicOr(status, ERR_TIMEOUT);
        tc::mbar_wait(&bars[0], (uint32_t)((nchunks - 1) & 1));
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, TC);
}

template <int PARTS>
static cudaError_t launch_parts(PtrArg p, Src src, int K, int n, long long ld, int B, const GramPlan& gp, ScaleArg sc,
                                float* P, int* status, cudaStream_t st) {
    constexpr int smem = smem_bytes<PARTS>();
    cudaError_t e = cudaFuncSetAttribute(k_gram_tc<PARTS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k_gram_tc<PARTS><<<dim3(gp.tiles, gp.S, B), NT, smem, st>>>(p, src, K, n, ld, gp, sc, P, status);
    return cudaGetLastError();
}

cudaError_t launch_gram_tc(PtrArg p, Src src, int K, int n, long long ld, int B, const GramPlan& gp, ScaleArg sc,
                           int accurate, float* P, int* status, cudaStream_t st) {
    if (accurate == GRAM_ACCURATE) return launch_parts<3>(p, src, K, n, ld, B, gp, sc, P, status, st);
    if (accurate == GRAM_DRAINED) return launch_parts<2>(p, src, K, n, ld, B, gp, sc, P, status, st);
    cudaError_t e = cudaFuncSetAttribute(k_gram_tc_plain, cudaFuncAttributeMaxDynamicSharedMemorySize, PLAIN_SMEM);
    if (e != cudaSuccess) return e;
    k_gram_tc_plain<<<dim3(gp.tiles, gp.S, B), PLAIN_NT, PLAIN_SMEM, st>>>(p, src, K, n, ld, gp, sc, P, status);
    return cudaGetLastError();
}

}  // namespace spq
