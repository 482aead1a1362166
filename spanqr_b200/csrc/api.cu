// C ABI of libspanqr: argument checks, workspace layout and the orth pass sequence.
//
// orth(X) (candidates/kcholqr.py:92-112, kcholqr_f with eps 5e-7, alpha 1e-7, tau 1e-8, ns 2) as a stream-ordered
// sequence of kernels; no host synchronisation, no device allocation.  Between passes Y lives in Q (the row-block
// kernels run in place), so the workspace holds only r x r matrices and the Gram partials.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/spanqr.h"
#include "kernels.h"

using namespace spq;

namespace {

constexpr float EPS = 5e-7f;    // dust weight, pass 1 (kcholqr.py:92)
constexpr int NS_STEPS = 2;     // Newton-Schulz polish steps (kcholqr.py:92)
constexpr int PASSES = 3;       // shifted Cholesky-QR passes (kcholqr.py:105)

thread_local char g_cuda_err[256] = "";

int cuda_fail(cudaError_t e) {
    std::snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
    return SPANQR_ERR_CUDA;
}

// ---- optional per-kernel timing (spanqr_timing_*) ----
enum Kind { K_SETUP = 0, K_ABSMAX, K_GRAM, K_REDUCE, K_CHOL, K_TRSM_W, K_TRSM, K_NS, K_GRAM_ACC, K_COPY, K_BAND, K_PROJ, K_COUNT };
const char* const KIND_NAMES[K_COUNT] = {"k_setup", "k_absmax", "k_gram_tc", "k_gram_reduce", "k_chol", "k_trsm_w", "k_trsm",
                                         "k_ns_update", "k_gram_tc_acc", "k_scale_copy", "k_band_image", "k_project"};
struct TimedLaunch {
    int kind;
    cudaEvent_t a, b;
    int nk;   // kernels between the two events
};
thread_local int g_timing = 0;                    // 0 off, 1 events around every launch, 2 count launches only
thread_local std::vector<TimedLaunch> g_launches;
thread_local long long g_counts[K_COUNT] = {};
thread_local std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pooled_event() {
    if (!g_event_pool.empty()) {
        cudaEvent_t e = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}

// run `launch`, which issues `nk` kernels, bracketed by events (mode 1) or counted (mode 2) when timing is on
template <typename F>
cudaError_t timed(int kind, cudaStream_t st, F&& launch, int nk = 1) {
    if (!g_timing) return launch();
    if (g_timing == 2) {
        g_counts[kind] += nk;
        return launch();
    }
    TimedLaunch t{kind, pooled_event(), pooled_event(), nk};
    if (!t.a || !t.b) return launch();
    cudaEventRecord(t.a, st);
    const cudaError_t e = launch();
    cudaEventRecord(t.b, st);
    g_launches.push_back(t);
    return e;
}

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
    size_t status, ptrs, maxbits, scal, rowsq, G, L, Li, W, maps, nss, P, total;
};

Layout layout(int K, int r, int B) {
    const GramPlan gp = gram_tc_plan(K, r);
    Layout l;
    size_t o = 0;
    l.status = o;  o += al256(256);
    l.ptrs = o;    o += al256(sizeof(MatPtr) * (size_t)B);
    l.maxbits = o; o += al256(sizeof(uint32_t) * (size_t)B);
    l.scal = o;    o += al256(sizeof(PassScal) * (size_t)B * PASSES);
    l.rowsq = o;   o += al256(sizeof(double) * (size_t)B * r);
    l.G = o;       o += al256(sizeof(float) * (size_t)B * r * r);
    l.L = o;       o += al256(sizeof(float) * (size_t)B * r * r);
    l.Li = o;      o += al256(sizeof(float) * (size_t)B * r * TB);
    l.W = o;       o += al256(trsm_w_bytes(r) * (size_t)B);
    l.maps = o;    o += al256((size_t)TMAPS_PER_MATRIX * 128 * B);
    // r > 256: the solve's second-panel start, later the polish update's first half
    l.nss = o;     o += (r > 256) ? al256(sizeof(float) * (size_t)B * K * 256) : 0;
    // the Gram's split partials; the polish step's D image reuses them once they are reduced
    size_t pbytes = sizeof(float) * (size_t)B * gp.S * gp.tiles * GRAM_TILE * GRAM_TILE;
    if (ns_dimg_bytes(r) * B > pbytes) pbytes = ns_dimg_bytes(r) * B;
    l.P = o;       o += al256(pbytes);
    l.total = o;
    return l;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_shape(int K, int r, int B) {
    if (r < TB || r > MAX_R || r % TB != 0 || K < r || B < 1 || B > 65535) return SPANQR_ERR_SHAPE;
    if ((long long)K * r > (1LL << 31)) return SPANQR_ERR_SHAPE;
    return SPANQR_OK;
}

int check_ws(void* ws, size_t ws_bytes, int K, int r, int B) {
    if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return SPANQR_ERR_WORKSPACE;
    if (ws_bytes < layout(K, r, B).total) return SPANQR_ERR_WORKSPACE;
    return SPANQR_OK;
}

template <typename T>
T* at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(ws) + off); }

// The solve on the tensor cores: one panel for n <= 256; for n > 256 the first 8 blocks, the product of those with
// the W tiles below them (the second panel's start) and the second panel.
cudaError_t run_trsm(PtrArg p, Src src, int K, int n, long long ldq, int B, const char* maps, const float* Z,
                     long long ldz, ScaleArg sc, float eps, const char* W, float* scratch, int* status, cudaStream_t st) {
    const int nb = n / TB;
    if (nb <= 8)
        return timed(K_TRSM, st, [&] {
            return launch_trsm_tc(p, src, K, n, ldq, B, 0, nb, nullptr, maps, Z, ldz, sc, eps, W, status, st);
        });
    cudaError_t e = timed(K_TRSM, st, [&] {
        return launch_trsm_tc(p, src, K, n, ldq, B, 0, 8, nullptr, maps, Z, ldz, sc, eps, W, status, st);
    });
    if (e == cudaSuccess)
        e = timed(K_TRSM, st, [&] { return launch_trsm_panel_product(p, K, n, ldq, B, 8, nb - 8, maps, W, scratch, status, st); });
    if (e == cudaSuccess)
        e = timed(K_TRSM, st, [&] {
            return launch_trsm_tc(p, src, K, n, ldq, B, 8, nb - 8, scratch, maps, Z, ldz, sc, eps, W, status, st);
        });
    return e;
}

// The pass sequence of kcholqr_f for B matrices whose pointers are in the workspace table (filled by k_setup_*).
// Z: the dust, K x r with leading dimension ldz (r when 0).
int run_orth(int K, int r, int B, long long ldx, long long ldq, const float* Z, void* ws, cudaStream_t st,
             long long ldz = 0) {
    if (ldz == 0) ldz = r;
    const Layout l = layout(K, r, B);
    const GramPlan gp = gram_tc_plan(K, r);
    PtrArg p{at<MatPtr>(ws, l.ptrs), MatPtr{nullptr, nullptr}};
    int* status = at<int>(ws, l.status);
    uint32_t* maxbits = at<uint32_t>(ws, l.maxbits);
    PassScal* scal = at<PassScal>(ws, l.scal);
    double* rowsq = at<double>(ws, l.rowsq);
    float* G = at<float>(ws, l.G);
    float* Lm = at<float>(ws, l.L);
    float* Li = at<float>(ws, l.Li);
    char* W = at<char>(ws, l.W);
    char* maps = at<char>(ws, l.maps);
    float* P = at<float>(ws, l.P);
    cudaError_t e;
#define SPQ_TRY(call)                          \
    do {                                       \
        if ((e = (call)) != cudaSuccess) return cuda_fail(e); \
    } while (0)
    SPQ_TRY(timed(K_ABSMAX, st, [&] { return launch_absmax(p, K, r, ldx, B, maxbits, st); }));
    SPQ_TRY(timed(K_SETUP, st, [&] { return launch_tmaps(p, K, r, ldx, ldq, B, ws, maps, st); }));
    for (int pass = 0; pass < PASSES; ++pass) {
        const bool first = pass == 0;
        const ScaleArg sc = first ? ScaleArg{maxbits, nullptr} : ScaleArg{nullptr, nullptr};
        // every pass uses the two-way split (passes 2 and 3 are plain SGEMMs in the reference; pass 1's compensated
        // gram_f is matched closely enough by it: the robustness and span tests pass either way)
        SPQ_TRY(timed(K_GRAM, st, [&] {
            return r <= 256 ? launch_gram_ws(p, first ? SRC_X : SRC_Q, K, r, B, gp, maps, sc, P, status, st)
                            : launch_gram_tc(p, first ? SRC_X : SRC_Q, K, r, first ? ldx : ldq, B, gp, sc, GRAM_PLAIN, P, status,
                                             st);
        }));
        SPQ_TRY(timed(K_REDUCE, st, [&] { return launch_gram_reduce(P, r, B, gp, 0, G, rowsq, st); }));
        SPQ_TRY(timed(K_CHOL, st, [&] {
            return launch_chol(G, Lm, Li, r, B, rowsq, gram_sq_parts(gp), nullptr, scal + (size_t)pass * B, 0, st);
        }));
        SPQ_TRY(timed(K_TRSM_W, st, [&] { return launch_trsm_w(Lm, Li, r, B, W, st); }));
        SPQ_TRY(run_trsm(p, first ? SRC_X : SRC_Q, K, r, ldq, B, maps, first ? Z : nullptr, ldz, sc, first ? EPS : 0.0f, W,
                         at<float>(ws, l.nss), status, st));
    }
    for (int it = 0; it < NS_STEPS; ++it) {
        // the last polish step's Gram (gram_split, kcholqr.py:20) decides Q's final orthogonality, and with it the
        // span error on the dominant directions: it drains its large-term accumulator into fp64 every 128 rows
        const bool last = it == NS_STEPS - 1;
        SPQ_TRY(timed(last ? K_GRAM_ACC : K_GRAM, st, [&] {
            return (r <= 256 && !last)
                       ? launch_gram_ws(p, SRC_Q, K, r, B, gp, maps, ScaleArg{nullptr, nullptr}, P, status, st)
                       : launch_gram_tc(p, SRC_Q, K, r, ldq, B, gp, ScaleArg{nullptr, nullptr},
                                        last ? GRAM_DRAINED : GRAM_PLAIN, P, status, st);
        }));
        SPQ_TRY(timed(K_REDUCE, st, [&] { return launch_gram_reduce(P, r, B, gp, 1, G, nullptr, st); }));
        // tensor cores for n <= 256; wider rows keep the shared-memory row-block kernel
        SPQ_TRY(timed(K_NS, st, [&] {
            return launch_ns_ws(p, K, r, ldq, B, G, maps, reinterpret_cast<char*>(P), at<float>(ws, l.nss), status, st);
        }, 2));   // the operand image of D, then the update
    }
#undef SPQ_TRY
    return SPANQR_OK;
}

}  // namespace

extern "C" {

int spanqr_version(void) { return 100; }

const char* spanqr_strerror(int code) {
    switch (code) {
        case SPANQR_OK: return "ok";
        case SPANQR_ERR_SHAPE: return "unsupported shape (r must be a multiple of 32 in [32, 512], K >= r, 1 <= batch <= 65535)";
        case SPANQR_ERR_ARG: return "bad argument (null or not 16-byte aligned pointer, or bad leading dimension)";
        case SPANQR_ERR_WORKSPACE: return "workspace too small or not 256-byte aligned";
        case SPANQR_ERR_CUDA: return "CUDA error";
        case SPANQR_ERR_DEVICE: return "device reported a failure";
        case SPANQR_ERR_TOO_LARGE: return "shape needs more scratch than the no-allocation entry point's fixed 16 MiB array";
        default: return "unknown status";
    }
}

const char* spanqr_last_cuda_error(void) { return g_cuda_err; }

int spanqr_workspace_bytes(int K, int r, int batch, size_t* bytes) {
    if (!bytes) return SPANQR_ERR_ARG;
    const int rc = check_shape(K, r, batch);
    if (rc) return rc;
    *bytes = layout(K, r, batch).total;
    return SPANQR_OK;
}

int spanqr_orth_strided_f32(const float* X, long long ldx, long long strideX, float* Q, long long ldq,
                            long long strideQ, int K, int r, int batch, const float* Z, void* ws, size_t ws_bytes,
                            spanqr_stream_t stream) {
    int rc = check_shape(K, r, batch);
    if (rc) return rc;
    if (!X || !Q || !Z || !a16(X) || !a16(Q) || !a16(Z)) return SPANQR_ERR_ARG;
    if (ldx < r || ldq < r || ldx % 4 || ldq % 4) return SPANQR_ERR_ARG;
    if (batch > 1 && (strideX % 4 || strideQ % 4 || strideQ < (long long)(K - 1) * ldq + r)) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, K, r, batch))) return rc;
    const Layout l = layout(K, r, batch);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = timed(K_SETUP, st, [&] {
        return launch_setup_strided(at<MatPtr>(ws, l.ptrs), X, strideX, Q, strideQ, batch, at<uint32_t>(ws, l.maxbits),
                                    at<int>(ws, l.status), st);
    });
    if (e != cudaSuccess) return cuda_fail(e);
    return run_orth(K, r, batch, ldx, ldq, Z, ws, st);
}

int spanqr_orth_f32(const float* X, long long ldx, float* Q, long long ldq, int K, int r, const float* Z, void* ws,
                    size_t ws_bytes, spanqr_stream_t stream) {
    return spanqr_orth_strided_f32(X, ldx, 0, Q, ldq, 0, K, r, 1, Z, ws, ws_bytes, stream);
}

int spanqr_orth_batched_f32(const float* const* dX, float* const* dQ, int K, int r, int batch, const float* Z,
                            void* ws, size_t ws_bytes, spanqr_stream_t stream) {
    int rc = check_shape(K, r, batch);
    if (rc) return rc;
    if (!dX || !dQ || !Z || !a16(Z)) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, K, r, batch))) return rc;
    const Layout l = layout(K, r, batch);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = timed(K_SETUP, st, [&] {
        return launch_setup_array(at<MatPtr>(ws, l.ptrs), dX, dQ, batch, at<uint32_t>(ws, l.maxbits),
                                  at<int>(ws, l.status), st);
    });
    if (e != cudaSuccess) return cuda_fail(e);
    return run_orth(K, r, batch, r, r, Z, ws, st);
}

int spanqr_orth_ptrs_f32(const float* const* hX, float* const* hQ, int K, int r, int batch, const float* Z, void* ws,
                         size_t ws_bytes, spanqr_stream_t stream) {
    int rc = check_shape(K, r, batch);
    if (rc) return rc;
    if (!hX || !hQ || !Z || !a16(Z)) return SPANQR_ERR_ARG;
    for (int b = 0; b < batch; ++b)
        if (!hX[b] || !hQ[b] || !a16(hX[b]) || !a16(hQ[b])) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, K, r, batch))) return rc;
    const Layout l = layout(K, r, batch);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = timed(K_SETUP, st, [&] {
        return launch_setup_host(at<MatPtr>(ws, l.ptrs), hX, hQ, batch, at<uint32_t>(ws, l.maxbits),
                                 at<int>(ws, l.status), st);
    }, setup_host_launches(batch));
    if (e != cudaSuccess) return cuda_fail(e);
    return run_orth(K, r, batch, r, r, Z, ws, st);
}

}  // extern "C"

// ---- a batch of matrices of one width and different heights ----
// Matrices are grouped by K in order of first appearance; group g runs as one batched orth over its own slice of the
// workspace, the groups one after another on the stream.  Each matrix gets the bits of a lone spanqr_orth_f32 call.
namespace {
struct KGroups {
    std::vector<int> K;                 // distinct heights, in order of first appearance
    std::vector<std::vector<int>> idx;  // the matrices of each height, in index order
};

int group_by_K(const int* K, int r, int batch, KGroups& g) {
    if (!K || batch < 1) return SPANQR_ERR_SHAPE;
    for (int b = 0; b < batch; ++b) {
        size_t i = 0;
        while (i < g.K.size() && g.K[i] != K[b]) ++i;
        if (i == g.K.size()) {
            g.K.push_back(K[b]);
            g.idx.emplace_back();
        }
        g.idx[i].push_back(b);
    }
    for (size_t i = 0; i < g.K.size(); ++i) {
        const int rc = check_shape(g.K[i], r, (int)g.idx[i].size());
        if (rc) return rc;
    }
    return SPANQR_OK;
}

size_t mixed_bytes(const KGroups& g, int r) {
    size_t t = 0;
    for (size_t i = 0; i < g.K.size(); ++i) t += al256(layout(g.K[i], r, (int)g.idx[i].size()).total);
    return t;
}
}  // namespace

extern "C" {

int spanqr_workspace_bytes_mixed(const int* K, int r, int batch, size_t* bytes) {
    if (!bytes) return SPANQR_ERR_ARG;
    KGroups g;
    const int rc = group_by_K(K, r, batch, g);
    if (rc) return rc;
    *bytes = mixed_bytes(g, r);
    return SPANQR_OK;
}

int spanqr_orth_mixed_f32(const float* const* hX, float* const* hQ, const int* K, int r, int batch,
                          const float* const* Z, void* ws, size_t ws_bytes, spanqr_stream_t stream) {
    KGroups g;
    int rc = group_by_K(K, r, batch, g);
    if (rc) return rc;
    if (!hX || !hQ || !Z) return SPANQR_ERR_ARG;
    for (size_t i = 0; i < g.K.size(); ++i)
        for (int b : g.idx[i])   // one dust per height
            if (!Z[b] || Z[b] != Z[g.idx[i][0]]) return SPANQR_ERR_ARG;
    if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0 || ws_bytes < mixed_bytes(g, r)) return SPANQR_ERR_WORKSPACE;
    char* w = static_cast<char*>(ws);
    std::vector<const float*> xs;
    std::vector<float*> qs;
    for (size_t i = 0; i < g.K.size(); ++i) {
        const int Bg = (int)g.idx[i].size();
        xs.clear();
        qs.clear();
        for (int b : g.idx[i]) {
            xs.push_back(hX[b]);
            qs.push_back(hQ[b]);
        }
        const size_t need = al256(layout(g.K[i], r, Bg).total);
        rc = spanqr_orth_ptrs_f32(xs.data(), qs.data(), g.K[i], r, Bg, Z[g.idx[i][0]], w, need, stream);
        if (rc) return rc;
        w += need;
    }
    return SPANQR_OK;
}

}  // extern "C"

// ---- orth as one CUDA graph per shape, X and Q patched per launch ----
// Every kernel of an orth call reads the matrix pointers from the workspace table except the set-up kernel, which
// writes them there: so a graph captured once per (K, r, ldx, ldq, Z, workspace) serves any X and Q after its set-up
// node's arguments are replaced (cudaGraphExecKernelNodeSetParams affects only launches made after it).
struct spanqr_graph_st {
    int dev, K, r;
    long long ldx, ldq;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    cudaGraphNode_t setup;
    cudaKernelNodeParams base;   // the set-up node as captured (function, launch shape)
    MatPtr* tab;
    uint32_t* maxbits;
    int* status;
};

extern "C" {

int spanqr_orth_graph_create(int K, int r, long long ldx, long long ldq, const float* Z, void* ws, size_t ws_bytes,
                             spanqr_graph_t* out) {
    if (!out) return SPANQR_ERR_ARG;
    *out = nullptr;
    int rc = check_shape(K, r, 1);
    if (rc) return rc;
    if (!Z || !a16(Z) || ldx < r || ldq < r || ldx % 4 || ldq % 4) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, K, r, 1))) return rc;
    const Layout l = layout(K, r, 1);
    spanqr_graph_st g{};
    g.K = K;
    g.r = r;
    g.ldx = ldx;
    g.ldq = ldq;
    g.tab = at<MatPtr>(ws, l.ptrs);
    g.maxbits = at<uint32_t>(ws, l.maxbits);
    g.status = at<int>(ws, l.status);
    cudaError_t e = cudaGetDevice(&g.dev);
    if (e != cudaSuccess) return cuda_fail(e);
    cudaStream_t cs = nullptr;
    if ((e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking)) != cudaSuccess) return cuda_fail(e);
    const int timing = g_timing;
    g_timing = 0;   // no timing events inside the graph
    e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        // the workspace stands in for X and Q until the first launch replaces them
        cudaError_t le = launch_setup_strided(g.tab, static_cast<const float*>(ws), 0, static_cast<float*>(ws), 0, 1,
                                              g.maxbits, g.status, cs);
        rc = (le == cudaSuccess) ? run_orth(K, r, 1, ldx, ldq, Z, ws, cs) : cuda_fail(le);
        e = cudaStreamEndCapture(cs, &g.graph);
        if (rc == SPANQR_OK && e != cudaSuccess) rc = cuda_fail(e);
    } else {
        rc = cuda_fail(e);
    }
    g_timing = timing;
    cudaStreamDestroy(cs);
    if (rc == SPANQR_OK) {
        size_t nn = 0;
        e = cudaGraphGetNodes(g.graph, nullptr, &nn);
        std::vector<cudaGraphNode_t> nodes(nn);
        if (e == cudaSuccess && nn) e = cudaGraphGetNodes(g.graph, nodes.data(), &nn);
        for (size_t i = 0; e == cudaSuccess && i < nn && !g.setup; ++i) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nodes[i], &t) != cudaSuccess || t != cudaGraphNodeTypeKernel) continue;
            cudaKernelNodeParams kp{};
            if (cudaGraphKernelNodeGetParams(nodes[i], &kp) == cudaSuccess && kp.func == setup_strided_kernel()) {
                g.setup = nodes[i];
                g.base = kp;
            }
        }
        if (e == cudaSuccess && !g.setup) e = cudaErrorNotSupported;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&g.exec, g.graph, 0);
        if (e != cudaSuccess) rc = cuda_fail(e);
    }
    if (rc != SPANQR_OK) {
        if (g.graph) cudaGraphDestroy(g.graph);
        return rc;
    }
    *out = new spanqr_graph_st(g);
    return SPANQR_OK;
}

int spanqr_orth_graph_launch(spanqr_graph_t g, const float* X, long long ldx, float* Q, long long ldq,
                             spanqr_stream_t stream) {
    if (!g || !X || !Q || !a16(X) || !a16(Q) || ldx != g->ldx || ldq != g->ldq) return SPANQR_ERR_ARG;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev != g->dev) return SPANQR_ERR_ARG;
    MatPtr* tab = g->tab;
    const float* x = X;
    float* q = Q;
    long long stride = 0;
    int B = 1;
    uint32_t* maxbits = g->maxbits;
    int* status = g->status;
    void* args[8] = {&tab, &x, &stride, &q, &stride, &B, &maxbits, &status};   // k_setup_strided's parameters
    cudaKernelNodeParams p = g->base;
    p.kernelParams = args;
    p.extra = nullptr;
    e = cudaGraphExecKernelNodeSetParams(g->exec, g->setup, &p);
    if (e == cudaSuccess) e = cudaGraphLaunch(g->exec, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_orth_graph_destroy(spanqr_graph_t g) {
    if (!g) return SPANQR_OK;
    cudaError_t e = cudaGraphExecDestroy(g->exec);
    const cudaError_t e2 = cudaGraphDestroy(g->graph);
    delete g;
    if (e == cudaSuccess) e = e2;
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

}  // extern "C"

// ---- block Gram-Schmidt for r > 512 (candidates/kbig.py:66-95, BCGS2 over 256-column blocks) ----
// Per block j (columns j .. j + 255): W = s X[:, j:j+256] is copied into Q's block (s = pow2_scale(max |X|) of the
// whole X), has the span of the finished blocks P = Q[:, :j] removed twice (W <- W - P (P^T W): a band Gram, -T as an
// operand image, the in-place tensor-core update), is orthonormalised in place by the orth sequence at width 256 with
// the dust's own 256 columns, and, for j > 0, is projected and orthonormalised once more.  The workspace starts with
// the orth layout of (K, 256, 1), so its status word is the one spanqr_read_status reads; the set-ups of the later
// blocks' orth sequences keep it.
namespace {
struct BorthLayout {
    size_t maxbits, maps, P, img, total;
};

BorthLayout borth_layout(int K, int r) {
    BorthLayout l;
    size_t o = al256(layout(K, BLOCK_W, 1).total);
    l.maxbits = o; o += 256;
    l.maps = o;    o += al256((size_t)TMAPS_PER_MATRIX * 128);
    size_t pb = 0;
    for (int j = BLOCK_W; j < r; j += BLOCK_W) {
        const GramPlan gp = gram_band_plan(K, j);
        const size_t b = sizeof(float) * (size_t)gp.S * gp.tiles * GRAM_TILE * GRAM_TILE;
        if (b > pb) pb = b;
    }
    l.P = o;       o += al256(pb);
    l.img = o;     o += al256(r > BLOCK_W ? band_img_bytes(r - BLOCK_W) : 0);
    l.total = o;
    return l;
}

constexpr int BORTH_MAX_R = 16384;

int check_borth_shape(int K, int r) {
    if (r < BLOCK_W || r > BORTH_MAX_R || r % BLOCK_W || K < r) return SPANQR_ERR_SHAPE;
    return check_shape(K, BLOCK_W, 1);
}

// W <- W - P (P^T W) for the block at column j of Q, in place
int project(float* Q, long long ldq, int K, int j, const char* maps, float* P, char* img, int* status, cudaStream_t st) {
    const GramPlan gp = gram_band_plan(K, j);
    const PtrArg q{nullptr, MatPtr{Q, Q}};
    cudaError_t e = timed(K_GRAM, st, [&] {
        return launch_gram_tc(q, SRC_Q, K, j + BLOCK_W, ldq, 1, gp, ScaleArg{nullptr, nullptr}, GRAM_PLAIN, P, status, st);
    });
    if (e == cudaSuccess) e = timed(K_BAND, st, [&] { return launch_band_image(P, gp, j, img, st); });
    if (e == cudaSuccess) e = timed(K_PROJ, st, [&] { return launch_project(q, K, j + BLOCK_W, ldq, j, maps, img, status, st); });
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

// the orth sequence at width 256, in place on Q's block at column j, with the dust's columns j .. j + 255
int block_orth(float* Q, long long ldq, int K, int j, const float* Z, long long ldz, void* ws, cudaStream_t st) {
    const Layout l = layout(K, BLOCK_W, 1);
    cudaError_t e = timed(K_SETUP, st, [&] {
        return launch_setup_strided(at<MatPtr>(ws, l.ptrs), Q + j, 0, Q + j, 0, 1, at<uint32_t>(ws, l.maxbits), nullptr, st);
    });
    if (e != cudaSuccess) return cuda_fail(e);
    return run_orth(K, BLOCK_W, 1, ldq, ldq, Z + j, ws, st, ldz);
}
}  // namespace

extern "C" {

int spanqr_workspace_bytes_borth(int K, int r, size_t* bytes) {
    if (!bytes) return SPANQR_ERR_ARG;
    const int rc = check_borth_shape(K, r);
    if (rc) return rc;
    *bytes = borth_layout(K, r).total;
    return SPANQR_OK;
}

int spanqr_borth_f32(const float* X, long long ldx, float* Q, long long ldq, int K, int r, const float* Z, void* ws,
                     size_t ws_bytes, spanqr_stream_t stream) {
    int rc = check_borth_shape(K, r);
    if (rc) return rc;
    if (!X || !Q || !Z || !a16(X) || !a16(Q) || !a16(Z)) return SPANQR_ERR_ARG;
    if (ldx < r || ldq < r || ldx % 4 || ldq % 4) return SPANQR_ERR_ARG;
    {   // Q is written while X is still read: the two must not overlap
        const uintptr_t x0 = reinterpret_cast<uintptr_t>(X), x1 = x0 + sizeof(float) * ((size_t)(K - 1) * ldx + r);
        const uintptr_t q0 = reinterpret_cast<uintptr_t>(Q), q1 = q0 + sizeof(float) * ((size_t)(K - 1) * ldq + r);
        if (x0 < q1 && q0 < x1) return SPANQR_ERR_ARG;
    }
    const BorthLayout bl = borth_layout(K, r);
    if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0 || ws_bytes < bl.total) return SPANQR_ERR_WORKSPACE;
    const Layout l = layout(K, BLOCK_W, 1);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int* status = at<int>(ws, l.status);
    uint32_t* maxall = at<uint32_t>(ws, bl.maxbits);
    char* maps = at<char>(ws, bl.maps);
    float* P = at<float>(ws, bl.P);
    char* img = at<char>(ws, bl.img);
    const PtrArg x{nullptr, MatPtr{X, Q}};
    cudaError_t e = timed(K_SETUP, st, [&] {
        return launch_setup_strided(at<MatPtr>(ws, l.ptrs), X, 0, Q, 0, 1, maxall, status, st);
    });
    if (e == cudaSuccess) e = timed(K_ABSMAX, st, [&] { return launch_absmax(x, K, r, ldx, 1, maxall, st); });
    if (e != cudaSuccess) return cuda_fail(e);
    for (int j = 0; j < r; j += BLOCK_W) {
        e = timed(K_COPY, st, [&] { return launch_scale_copy(X + j, ldx, Q + j, ldq, K, BLOCK_W, maxall, st); });
        if (e == cudaSuccess && j > 0)
            e = timed(K_SETUP, st, [&] { return launch_tmaps(PtrArg{nullptr, MatPtr{Q, Q}}, K, j, ldq, ldq, 1, ws, maps, st); });
        if (e != cudaSuccess) return cuda_fail(e);
        for (int t = 0; j > 0 && t < 2; ++t)
            if ((rc = project(Q, ldq, K, j, maps, P, img, status, st))) return rc;
        if ((rc = block_orth(Q, ldq, K, j, Z, r, ws, st))) return rc;
        if (j > 0) {
            if ((rc = project(Q, ldq, K, j, maps, P, img, status, st))) return rc;
            if ((rc = block_orth(Q, ldq, K, j, Z, r, ws, st))) return rc;
        }
    }
    return SPANQR_OK;
}

}  // extern "C"

// ---- orth without any allocation: scratch in a fixed array of the device image ----
// For callers that may not call cudaMalloc (inside a stream capture that must not add allocations, in a
// memory-capped sandbox, in a real-time loop).  The array belongs to the library's module: each GPU that loads the
// library keeps it until the process exits.  Its host-side name is only a stand-in, never a device address; the
// device address is looked up with cudaGetSymbolAddress once per device and context (a cudaDeviceReset gives the
// device a new context, and with it a new copy of the array, so the cached address is keyed on the context too).
namespace {
static __device__ __align__(256) unsigned char g_noalloc_scratch[SPANQR_NOALLOC_SCRATCH_BYTES];
constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
struct NoallocSlot {
    void* ctx;
    void* ptr;
};
NoallocSlot g_noalloc[NOALLOC_MAX_DEVICES] = {};

using CtxGetCurrentFn = int (*)(void**);   // cuCtxGetCurrent(CUcontext*)
CtxGetCurrentFn g_ctx_get = nullptr;
std::once_flag g_ctx_once;

// the scratch array's device address for the current device and context (looked up on first use)
int noalloc_scratch(void** out) {
    std::call_once(g_ctx_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 4000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_get = reinterpret_cast<CtxGetCurrentFn>(fn);
    });
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return SPANQR_ERR_ARG;
    void* ctx = nullptr;
    if (!g_ctx_get || g_ctx_get(&ctx) != 0) return cuda_fail(cudaErrorNotSupported);
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!ctx || !g_noalloc[dev].ptr || g_noalloc[dev].ctx != ctx) {
        // with device `dev` current; the lookup also makes the device's primary context current if none was
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e);
        if (g_ctx_get(&ctx) != 0 || !ctx) return cuda_fail(cudaErrorNotSupported);
        g_noalloc[dev] = NoallocSlot{ctx, p};
    }
    *out = g_noalloc[dev].ptr;
    return SPANQR_OK;
}
}  // namespace

extern "C" {

int spanqr_orth_noalloc_f32(const float* X, long long ldx, float* Q, long long ldq, int K, int r, const float* Z,
                            spanqr_stream_t stream) {
    int rc = check_shape(K, r, 1);
    if (rc) return rc;
    if (layout(K, r, 1).total > SPANQR_NOALLOC_SCRATCH_BYTES) return SPANQR_ERR_TOO_LARGE;
    void* scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    // the set-up kernel of the orth sequence clears the only scratch words that must start at zero (the per-matrix
    // max |x| bits and the status word); every other scratch region is fully written before it is read
    return spanqr_orth_f32(X, ldx, Q, ldq, K, r, Z, scratch, SPANQR_NOALLOC_SCRATCH_BYTES, stream);
}

int spanqr_noalloc_read_status(spanqr_stream_t stream, int* device_status) {
    if (!device_status) return SPANQR_ERR_ARG;
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    return spanqr_read_status(scratch, stream, device_status);   // the status word leads the scratch layout
}

int spanqr_gram_f32(const float* Y, long long ldy, int K, int n, const float* d_s, float* G, void* ws,
                    size_t ws_bytes, spanqr_stream_t stream) {
    int rc = check_shape(K, n, 1);
    if (rc) return rc;
    if (!Y || !G || !a16(Y) || ldy < n || ldy % 4) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, K, n, 1))) return rc;
    const Layout l = layout(K, n, 1);
    const GramPlan gp = gram_tc_plan(K, n);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    PtrArg p{nullptr, MatPtr{Y, nullptr}};
    cudaError_t e = cudaMemsetAsync(at<int>(ws, l.status), 0, sizeof(int), st);
    if (e == cudaSuccess)
        e = launch_gram_tc(p, SRC_X, K, n, ldy, 1, gp, ScaleArg{nullptr, d_s}, GRAM_ACCURATE, at<float>(ws, l.P),
                           at<int>(ws, l.status), st);
    if (e == cudaSuccess) e = launch_gram_reduce(at<float>(ws, l.P), n, 1, gp, 0, G, nullptr, st);
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_gram_mode_f32(const float* Y, long long ldy, int K, int n, const float* d_s, int mode, float* G, void* ws,
                         size_t ws_bytes, spanqr_stream_t stream) {
    if (mode == SPANQR_GRAM_ACCURATE) return spanqr_gram_f32(Y, ldy, K, n, d_s, G, ws, ws_bytes, stream);
    if (mode != SPANQR_GRAM_PASS && mode != SPANQR_GRAM_POLISH) return SPANQR_ERR_ARG;
    int rc = check_shape(K, n, 1);
    if (rc) return rc;
    if (!Y || !G || !a16(Y) || ldy < n || ldy % 4) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, K, n, 1))) return rc;
    const Layout l = layout(K, n, 1);
    const GramPlan gp = gram_tc_plan(K, n);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    PtrArg p{nullptr, MatPtr{Y, const_cast<float*>(Y)}};
    const ScaleArg sc{nullptr, d_s};
    int* status = at<int>(ws, l.status);
    float* P = at<float>(ws, l.P);
    cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), st);
    if (e == cudaSuccess && mode == SPANQR_GRAM_PASS && n <= 256)
        e = launch_tmaps(p, K, n, ldy, ldy, 1, ws, at<char>(ws, l.maps), st);
    if (e == cudaSuccess) {
        if (mode == SPANQR_GRAM_PASS)   // the Gram of every Cholesky-QR pass and of the first polish step
            e = n <= 256 ? launch_gram_ws(p, SRC_X, K, n, 1, gp, at<char>(ws, l.maps), sc, P, status, st)
                         : launch_gram_tc(p, SRC_X, K, n, ldy, 1, gp, sc, GRAM_PLAIN, P, status, st);
        else   // the last polish step's Gram
            e = launch_gram_tc(p, SRC_X, K, n, ldy, 1, gp, sc, GRAM_DRAINED, P, status, st);
    }
    if (e == cudaSuccess) e = launch_gram_reduce(P, n, 1, gp, 0, G, nullptr, st);
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_chol_f32(const float* G, int n, const float* d_tau, float* L, float* Li, void* ws, size_t ws_bytes,
                    spanqr_stream_t stream) {
    int rc = check_shape(n, n, 1);
    if (rc) return rc;
    if (!G || !d_tau || !L || !Li) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, n, n, 1))) return rc;
    const Layout l = layout(n, n, 1);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    float* A = at<float>(ws, l.G);
    cudaError_t e = cudaMemcpyAsync(A, G, sizeof(float) * (size_t)n * n, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = launch_chol(A, L, Li, n, 1, nullptr, 0, d_tau, nullptr, 1, st);
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_trsm_f32(const float* X, long long ldx, const float* Z, const float* d_s, float eps, const float* L,
                    const float* Li, int K, int n, float* Y, long long ldy, void* ws, size_t ws_bytes,
                    spanqr_stream_t stream) {
    int rc = check_shape(K, n, 1);
    if (rc) return rc;
    if (!X || !Y || !L || !Li || !a16(X) || !a16(Y) || (Z && !a16(Z))) return SPANQR_ERR_ARG;
    if (ldx < n || ldy < n || ldx % 4 || ldy % 4) return SPANQR_ERR_ARG;
    if ((rc = check_ws(ws, ws_bytes, K, n, 1))) return rc;
    const Layout l = layout(K, n, 1);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    PtrArg p{nullptr, MatPtr{X, Y}};
    cudaError_t e = cudaMemsetAsync(at<int>(ws, l.status), 0, sizeof(int), st);
    if (e == cudaSuccess) e = launch_trsm_w(L, Li, n, 1, at<char>(ws, l.W), st);
    if (e == cudaSuccess) e = launch_tmaps(p, K, n, ldx, ldy, 1, ws, at<char>(ws, l.maps), st);
    if (e == cudaSuccess)
        e = run_trsm(p, SRC_X, K, n, ldy, 1, at<char>(ws, l.maps), Z, n, ScaleArg{nullptr, d_s}, Z ? eps : 0.0f,
                     at<char>(ws, l.W), at<float>(ws, l.nss), at<int>(ws, l.status), st);
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_timing_enable(int mode) {
    if (mode < 0 || mode > 2) return SPANQR_ERR_ARG;
    g_timing = mode;
    return SPANQR_OK;
}

int spanqr_timing_collect(double* ms, long long* launches, int nkinds) {
    if ((!ms || !launches) && nkinds > 0) return SPANQR_ERR_ARG;
    int rc = SPANQR_OK;
    for (const TimedLaunch& t : g_launches) {
        float dt = 0.0f;
        cudaError_t e = cudaEventSynchronize(t.b);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&dt, t.a, t.b);
        if (e != cudaSuccess) rc = cuda_fail(e);
        else if (t.kind < nkinds) {
            ms[t.kind] += dt;
            launches[t.kind] += t.nk;
        }
        g_event_pool.push_back(t.a);
        g_event_pool.push_back(t.b);
    }
    g_launches.clear();
    for (int k = 0; k < K_COUNT; ++k) {
        if (k < nkinds) launches[k] += g_counts[k];
        g_counts[k] = 0;
    }
    return rc;
}

int spanqr_kernel_kinds(void) { return K_COUNT; }

const char* spanqr_kernel_kind_name(int kind) { return (kind >= 0 && kind < K_COUNT) ? KIND_NAMES[kind] : ""; }

int spanqr_selftest_timeout(void* ws, size_t ws_bytes, long long limit_ns, int arrive, spanqr_stream_t stream) {
    if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0 || ws_bytes < 256) return SPANQR_ERR_WORKSPACE;
    if (limit_ns <= 0 || limit_ns > 2000000000LL) return SPANQR_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(int), st);
    if (e == cudaSuccess) e = launch_wait_selftest(arrive != 0, (unsigned long long)limit_ns, static_cast<int*>(ws), st);
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

// ---- exchange slabs of orth_batched across the GPUs of one node (no reference counterpart) ----
static_assert(sizeof(cudaIpcMemHandle_t) == SPANQR_PEER_HANDLE_BYTES, "IPC handle size");

int spanqr_peer_slab_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle || bytes == 0) return SPANQR_ERR_ARG;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e);
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e);
    }
    std::memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return SPANQR_OK;
}

int spanqr_peer_slab_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return SPANQR_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e);
    *ptr = p;
    return SPANQR_OK;
}

int spanqr_peer_slab_close(void* ptr) {
    if (!ptr) return SPANQR_ERR_ARG;
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_peer_slab_free(void* ptr) {
    if (!ptr) return SPANQR_ERR_ARG;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_peer_copy(void* dst, const void* src, size_t bytes, spanqr_stream_t stream) {
    if (bytes == 0) return SPANQR_OK;
    if (!dst || !src) return SPANQR_ERR_ARG;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SPANQR_OK : cuda_fail(e);
}

int spanqr_read_status(const void* ws, spanqr_stream_t stream, int* device_status) {
    if (!ws || !device_status) return SPANQR_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, ws, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e);
    *device_status = h;
    return h ? SPANQR_ERR_DEVICE : SPANQR_OK;
}

}  // extern "C"
