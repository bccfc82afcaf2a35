// model.cu — the PP-DocLayoutV3 forward on one B200 and the public C ABI
// of include/ppdoclayout.h.
//
// The reference builds a ggml graph of ~1000-1700 nodes and runs it with
// ggml_backend_sched + CUDA-graph replay (src/ppdoclayout.cpp:733-882,
// 1082-1191).  Here the same network is a static plan of kernel launches
// built once at init for a batch capacity B (pages), captured into one CUDA
// graph per batch size and replayed:
//
//   * every conv goes through conv() — the reference's builder::conv
//     dispatch (src/ppdoclayout.cpp:388-543): depthwise -> direct kernel;
//     1x1 -> GEMM writing CHW (bias + activation fused); k3-s1-p1 ->
//     Winograd F(4,3); k3-s2 and k2 -> implicit GEMM fed by TMA windows of
//     the input (no im2col buffer);
//   * concatenations are free: producers write straight into channel
//     slices of the consumer's buffer (HG-block aggregation, CCFM/PAN
//     concats), and residual adds ride in the producing epilogue;
//   * all pages of a batch run in the same launches (page stride per view);
//   * the two-stage selection, decoder, heads and the postprocess stay on
//     the device; only the image goes in and dets + masks come out.
//
// Buffers are allocated once per context (no aliasing: activation memory is
// ~0.8 GB per page against 180 GB of HBM).
#include <cuda_runtime.h>
#include <sys/stat.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/ppdoclayout.h"
#include "common.cuh"
#include "conv.h"
#include "dec.h"
#include "gemm.h"
#include "gemm_tc.h"
#include "gguf.h"
#include "kernels.h"

namespace ppdl {

namespace {

struct WT {
    float *p = nullptr;
    int64_t ne[4] = {1, 1, 1, 1};
};

// CHW activation view: page b, channel c at p + b*bs + c*H*W
struct V {
    float *p = nullptr;
    int C = 0, H = 0, W = 0;
    long long bs = 0;
    long long plane() const { return (long long)H * W; }
    V slice(int c0, int nc) const {
        V v = *this;
        v.p = p + (long long)c0 * H * W;
        v.C = nc;
        return v;
    }
};

// token-major activation [B][T][D] (contiguous)
struct S {
    float *p = nullptr;
    int T = 0, D = 0;
    long long bs() const { return (long long)T * D; }
};

struct Dump {
    std::string name;
    const void *p;
    int64_t ne[4];
    const char *type;
    size_t bytes;
};

// One launch group of the plan: a name, a kernel class (PPDL_STEP_*), the
// algorithmic FLOPs and bytes per page, and the closure that enqueues it.
// Steps run on lanes (streams) inside the forward: lane 0 is the context's
// stream; a step waits for the plan events in `waits` (each recorded after
// an earlier step of another lane) and records event `record` after itself.
// Latency-bound decoder launches that use a few dozen SMs then overlap with
// each other and with the value projections.
struct Step {
    std::string name;
    int kind;
    double flops, bytes;
    std::function<Status()> fn;
    int lane = 0;
    std::vector<int> waits;
    int record = -1;
};

constexpr int kLanes = 3;
#ifndef PPDL_VP_CTAS
#define PPDL_VP_CTAS 120
#endif
constexpr int kVpCtas = PPDL_VP_CTAS;  // SMs a value projection may hold (of 148)

#define TRY(x)                         \
    do {                               \
        Status s_ = (x);               \
        if (s_ != OK) return s_;       \
    } while (0)

}  // namespace

class Model {
public:
    int dev = 0, Bmax = 1, nb = 1;
    bool dumps = false;
    bool ok = true;
    std::string err;
    cudaStream_t st = nullptr;
    std::unordered_map<std::string, WT> w;
    std::vector<void *> allocs;
    std::vector<Step> plan;
    int lane = 0, lane_last[kLanes] = {-1, -1, -1}, n_events = 0;
    std::vector<int> pending;
    cudaStream_t lanes[kLanes] = {};
    std::vector<cudaEvent_t> events;  // n_events plan events + kLanes fork/join
    std::map<int, cudaGraphExec_t> graphs;
    std::vector<Dump> dump_list;

    // Winograd / attention scratch (sized while the plan is built)
    // Two scratch sets: set 1 serves the mask-feature head, which runs on a
    // side lane at the same time as set 0's users on lane 0.
    float *wg_dt_s[2] = {}, *wg_yt_s[2] = {};
    long long wg_dt_ns[2] = {}, wg_yt_ns[2] = {};
    int scratch = 0;  // set used by the convs planned next

    // graph inputs / outputs
    V img;
    int32_t *ori_hw = nullptr;
    S logits, boxes, order;
    float *dets = nullptr;
    int32_t *sel = nullptr, *rank = nullptr, *masks = nullptr;
    uint32_t *mask_bits = nullptr;  // packed masks [B][300][1250], made by the forward
    int32_t *enc_topk = nullptr;  // encoder top-300 token indices (query order)

    ~Model() {
        for (auto &g : graphs) cudaGraphExecDestroy(g.second);
        for (void *p : allocs) cudaFree(p);
        for (auto e : events) cudaEventDestroy(e);
        for (int l = 0; l < kLanes; l++)
            if (lanes[l]) cudaStreamDestroy(lanes[l]);
    }

    // Tensor-core (3xTF32) GEMMs for every contraction whose operands satisfy
    // the TMA rules; the SIMT FFMA GEMM takes the rest.  PPDL_TC=0 forces the
    // SIMT path everywhere (a bisection knob like the reference's
    // PPDL_CONV_MODE, src/ppdoclayout.cpp:392-398).
    bool use_tc = true;
    std::vector<std::function<void()>> finalizers;  // plans that need the scratch buffers

    struct Split {
        float *hi = nullptr, *lo = nullptr;
    };
    Split split(const float *w, long long n) {
        Split s;
        s.hi = dalloc(n);
        s.lo = dalloc(n);
        if (ok && launch_tf32_split(w, s.hi, s.lo, n, st) != OK) fail("weight split failed");
        return s;
    }
    static bool tc_shape_ok(const float *p, long long plane, long long bs, int K) {
        return ((uintptr_t)p & 15) == 0 && plane % 4 == 0 && bs % 4 == 0 && K % 4 == 0;
    }
    // Tensor-core conv of a k3-s2 / k2 kernel read straight from the CHW
    // input (implicit GEMM, no im2col buffer): TMA windows of the input
    // (box mode) when its rows are 16-byte multiples, else the converter
    // warps' gather.  Returns a null plan when neither applies (the caller
    // keeps the SIMT GEMM).
    std::shared_ptr<TcGemm> plan_conv_implicit(const V &x, int K, int s, int p, int OC, int OH,
                                               int OW, const float *wp, const TcEpilogue &e,
                                               const std::string &name) {
        if (!ok) return nullptr;
        auto g = std::make_shared<TcGemm>();
        TcConvBox cb;
        cb.x = x.p; cb.x_bs = x.bs;
        cb.IC = x.C; cb.H = x.H; cb.W = x.W; cb.KS = K; cb.S = s; cb.P = p;
        cb.OH = OH; cb.OW = OW;
        if (x.W % 4) {
            // rows that are not 16-byte multiples (a 50-wide input): the
            // windows come from a copy with rows padded to Wp = W rounded up
            // to 4 (zeros past W, which the conv reads as its padding)
            const int Wp = (x.W + 3) / 4 * 4;
            const long long pbs = (long long)x.C * x.H * Wp;
            float *xp = dalloc(pbs * Bmax);
            if (!ok) return nullptr;
            const V xv = x;
            push(name + ".pad_rows", PPDL_STEP_GLUE, 0.0,
                 4.0 * ((double)x.C * x.plane() + (double)pbs), [=]() {
                return launch_pad_rows(xv.p, xv.bs, xp, pbs, xv.C, xv.H, xv.W, Wp, nb, st);
            });
            cb.x = xp; cb.x_bs = pbs; cb.W = Wp;
        }
        const int Kb = tc_conv_box_kdim(x.C, K);
        float *hi = dalloc((long long)OC * Kb), *lo = dalloc((long long)OC * Kb);
        if (!ok) return nullptr;
        if (tc_gemm_plan_box(g.get(), OC, Bmax, cb, hi, lo, e)) {
            if (launch_tf32_split_box(wp, hi, lo, OC, x.C, K, st) != OK) {
                fail("weight split failed");
                return nullptr;
            }
            return g;
        }
        // gather: B = the raw weight rows [OC][IC*K*K] padded to 16 bytes
        const int Kc = x.C * K * K, Kp = (Kc + 3) / 4 * 4;
        if ((long long)Kp > Kb) {
            hi = dalloc((long long)OC * Kp);
            lo = dalloc((long long)OC * Kp);
            if (!ok) return nullptr;
        }
        TcGather gg;
        gg.x = x.p; gg.x_bs = x.bs; gg.plane = x.plane();
        gg.KS = K; gg.S = s; gg.P = p; gg.H = x.H; gg.W = x.W; gg.OW = OW;
        if (!tc_gemm_plan_gather(g.get(), OH * OW, OC, Kc, Bmax, gg, hi, lo, e)) return nullptr;
        if (launch_tf32_split_pad(wp, hi, lo, OC, Kc, Kp, st) != OK) {
            fail("weight split failed");
            return nullptr;
        }
        return g;
    }
    // Tensor-core 1x1 conv on planes that TMA cannot take as one tensor
    // (H*W not a multiple of 4, e.g. 25 x 25): A is loaded as per-channel
    // TMA rows (rows mode).  Null plan when even that does not apply.
    std::shared_ptr<TcGemm> plan_conv1x1_rows(const V &x, int OC, const float *wp,
                                              const TcEpilogue &e) {
        if (!ok || x.C % 4) return nullptr;
        const Split wsp = split(wp, (long long)OC * x.C);
        auto g = std::make_shared<TcGemm>();
        if (!ok || !tc_gemm_plan_rows(g.get(), (int)x.plane(), OC, x.C, Bmax, x.p, x.plane(), x.bs,
                                      wsp.hi, wsp.lo, e))
            return nullptr;
        return g;
    }
    // conv epilogue writing a CHW view
    static TcEpilogue chw_epilogue(const V &y, const float *bp, int act, const V &res,
                                   int res_mode) {
        TcEpilogue e;
        e.C = y.p; e.ldc_m = 1; e.ldc_n = y.plane(); e.c_bs = y.bs;
        e.bias = bp; e.act = act;
        if (res_mode) {
            e.res = res.p; e.res_ldm = 1; e.res_ldn = res.plane(); e.res_bs = res.bs;
            e.res_mode = res_mode;
        }
        return e;
    }
    // launch a planned tensor-core GEMM for the current batch: rows_per_page > 0
    // folds the pages into M (zmul z slices, e.g. the 36 Winograd planes),
    // otherwise every page (x zmul planes) is a z slice
    Status run_tc(const std::shared_ptr<TcGemm> &g, int rows_per_page, int zmul = 1) {
        TcGemm r = *g;
        if (rows_per_page > 0) {
            r.M = nb * rows_per_page;
            r.m_tiles = (r.M + 127) / 128;
            r.batch = zmul;
        } else {
            r.batch = nb * zmul;
        }
        r.tiles = r.m_tiles * r.n_tiles * r.batch;
        return launch_tc_gemm(r, st);
    }

    template <typename F>
    void push(const std::string &name, int kind, double flops, double bytes, F fn) {
        Step s{name, kind, flops, bytes, std::function<Status()>(fn)};
        s.lane = lane;
        s.waits.swap(pending);
        lane_last[lane] = (int)plan.size();
        plan.push_back(std::move(s));
    }
    // event recorded after the latest step of the current lane (all of that
    // lane's steps so far are done when it fires)
    int mark() {
        const int li = lane_last[lane];
        if (li < 0) {
            fail("mark on an empty lane");
            return 0;
        }
        if (plan[li].record < 0) plan[li].record = n_events++;
        return plan[li].record;
    }
    // the next step pushed on the current lane waits for event e
    void after(int e) { pending.push_back(e); }
    void on_lane(int l) {
        if (!pending.empty()) fail("lane switch with pending waits");
        lane = l;
    }

    void fail(const std::string &m) {
        if (ok) err = m;
        ok = false;
    }

    float *dalloc(long long nfloats) {
        void *p = nullptr;
        if (nfloats <= 0) nfloats = 1;
        if (cudaMalloc(&p, (size_t)nfloats * sizeof(float)) != cudaSuccess) {
            fail("cudaMalloc of " + std::to_string(nfloats * 4) + " bytes failed");
            return nullptr;
        }
        allocs.push_back(p);
        return (float *)p;
    }
    V tensor(int C, int H, int W) {
        V v;
        v.C = C; v.H = H; v.W = W;
        v.bs = (long long)C * H * W;
        v.p = dalloc(v.bs * Bmax);
        return v;
    }
    S seq(int T, int D) {
        S s;
        s.T = T; s.D = D;
        s.p = dalloc((long long)T * D * Bmax);
        return s;
    }
    const WT &W(const std::string &n) {
        static WT none;
        auto it = w.find(n);
        if (it == w.end()) {
            fail("missing tensor: " + n);
            return none;
        }
        return it->second;
    }
    void dump_chw(const char *name, const V &v) {
        if (dumps)
            dump_list.push_back({name, v.p, {v.W, v.H, v.C, 1}, "f32", (size_t)v.C * v.plane() * 4});
    }
    void dump_seq(const char *name, const S &s) {
        if (dumps) dump_list.push_back({name, s.p, {s.D, s.T, 1, 1}, "f32", (size_t)s.bs() * 4});
    }

    // ---- model loading (src/ppdoclayout.cpp:217-246) ------------------------
    bool load(const char *path) {
        GgufFile g;
        std::string e;
        if (!gguf_read_header(path, &g, &e)) {
            fail(e);
            return false;
        }
        size_t total = 0;
        for (auto &t : g.tensors) total += (t.nbytes + 255) / 256 * 256;
        float *base = dalloc((long long)(total / 4));
        if (!ok) return false;
        FILE *f = fopen(path, "rb");
        if (!f) {
            fail(std::string("cannot open ") + path);
            return false;
        }
        void *stage = nullptr;
        const size_t kStage = 64u << 20;
        if (cudaHostAlloc(&stage, kStage, cudaHostAllocDefault) != cudaSuccess) {
            fclose(f);
            fail("cudaHostAlloc failed");
            return false;
        }
        size_t off = 0;
        for (auto &t : g.tensors) {
            WT wt;
            wt.p = (float *)((char *)base + off);
            for (int d = 0; d < 4; d++) wt.ne[d] = t.ne[d];
            fseeko(f, (off_t)(g.data_offset + t.offset), SEEK_SET);
            size_t done = 0;
            while (done < t.nbytes) {
                const size_t n = std::min(kStage, (size_t)t.nbytes - done);
                if (fread(stage, 1, n, f) != n) {
                    fail("short read of tensor " + t.name);
                    break;
                }
                cudaMemcpy((char *)wt.p + done, stage, n, cudaMemcpyHostToDevice);
                done += n;
            }
            if (!ok) break;
            w[t.name] = wt;
            off += (t.nbytes + 255) / 256 * 256;
        }
        fclose(f);
        cudaFreeHost(stage);
        return ok;
    }

    // ---- conv dispatch (builder::conv, src/ppdoclayout.cpp:388-543) ---------
    // y = act(conv(x) + bias (+ res if res_mode == 1)) (+ res if res_mode == 2)
    // p_hi < 0: symmetric padding p; otherwise bottom/right padding p_hi
    // (the stem's ggml_pad, :621-624).
    // w_ov / b_ov: weight and bias tensors to use instead of the named ones
    // (folded or stacked weights; name then only names the step)
    void conv(const V &x, const V &y, const std::string &name, int s, int p, int act,
              const V &res = V(), int res_mode = 0, int p_hi = -1, const WT *w_ov = nullptr,
              const WT *b_ov = nullptr) {
        const WT &wt = w_ov ? *w_ov : W(name + ".weight");
        const WT &bt = b_ov ? *b_ov : W(name + ".bias");
        if (!ok) return;
        const int K = (int)wt.ne[0], IC = (int)wt.ne[2], OC = (int)wt.ne[3];
        const int ph = p_hi < 0 ? p : p_hi;
        const int OH = (x.H + p + ph - K) / s + 1, OW = (x.W + p + ph - K) / s + 1;
        const bool dw = IC == 1 && x.C != 1;
        if (wt.ne[1] != K || (dw ? OC != x.C : IC != x.C) || y.C != OC || y.H != OH || y.W != OW ||
            bt.ne[0] != OC) {
            fail("conv " + name + ": shape mismatch");
            return;
        }
        const float *wp = wt.p, *bp = bt.p;
        if (dw) {
            if (res_mode || p_hi >= 0) {
                fail("conv " + name + ": depthwise form not supported");
                return;
            }
            push(name, PPDL_STEP_DWCONV, 2.0 * OC * OH * OW * K * K,
                 4.0 * ((double)x.C * x.plane() + (double)OC * OH * OW + OC * K * K), [=]() {
                return launch_dwconv(x.p, x.bs, wp, bp, y.p, y.bs, x.C, x.H, x.W, K, s, p, act, nb,
                                     st);
            });
            return;
        }
        if (K == 1 && s == 1 && p == 0 && p_hi < 0) {
            // tensor cores: A = x (pixels x channels, M-major), B = W [OC][IC]
            if (use_tc && tc_shape_ok(x.p, x.plane(), x.bs, IC)) {
                const Split wsp = split(wp, (long long)OC * IC);
                TcEpilogue e;
                e.C = y.p; e.ldc_m = 1; e.ldc_n = y.plane(); e.c_bs = y.bs;
                e.bias = bp; e.act = act;
                if (res_mode) {
                    e.res = res.p; e.res_ldm = 1; e.res_ldn = res.plane(); e.res_bs = res.bs;
                    e.res_mode = res_mode;
                }
                auto g = std::make_shared<TcGemm>();
                if (ok && tc_gemm_plan(g.get(), (int)x.plane(), OC, IC, Bmax, x.p, 1, x.plane(),
                                       x.bs, wsp.hi, wsp.lo, 1, e)) {
                    push(name, PPDL_STEP_GEMM_1X1, 2.0 * OC * OH * OW * IC,
                         4.0 * ((double)IC * x.plane() + (double)OC * OH * OW),
                         [=]() { return run_tc(g, 0); });
                    return;
                }
            } else if (use_tc) {
                auto g = plan_conv1x1_rows(x, OC, wp, chw_epilogue(y, bp, act, res, res_mode));
                if (g) {
                    push(name, PPDL_STEP_GEMM_1X1, 2.0 * OC * OH * OW * IC,
                         4.0 * ((double)IC * x.plane() + (double)OC * OH * OW),
                         [=]() { return run_tc(g, 0); });
                    return;
                }
            }
            push(name, PPDL_STEP_GEMM_1X1, 2.0 * OC * OH * OW * IC,
                 4.0 * ((double)IC * x.plane() + (double)OC * OH * OW), [=]() {
                GemmArgs g;
                g.M = OC; g.N = OH * OW; g.K = IC; g.batch = nb;
                g.A = {wp, IC, 1};
                g.B = {x.p, x.plane(), 1, 1, x.bs, 0};
                g.C = y.p; g.ldc_m = y.plane(); g.ldc_n = 1; g.c_bs_hi = y.bs;
                g.bias = bp; g.bias_mode = 1; g.act = act;
                if (res_mode) {
                    g.res = {res.p, res.plane(), 1, 1, res.bs, 0};
                    g.res_mode = res_mode;
                }
                return launch_gemm_simt(g, st);
            });
            return;
        }
        if (K == 3 && s == 1 && p == 1 && p_hi < 0) {
            // Winograd F(4,3) (src/ppdoclayout.cpp:430-464)
            // plane rows padded to 4 floats so TMA row strides are 16-byte multiples
            const int TW = (x.W + 3) / 4, TH = (x.H + 3) / 4, T = TW * TH;
            const int Tp = (T + 3) / 4 * 4;
            float *wg4 = dalloc(36LL * IC * OC);
            if (!ok) return;
            if (launch_wg4_filter(wp, wg4, IC, OC, st) != OK) {
                fail("filter transform launch failed");
                return;
            }
            const int ss = scratch;
            wg_dt_ns[ss] = std::max(wg_dt_ns[ss], 36LL * IC * Tp * Bmax);
            wg_yt_ns[ss] = std::max(wg_yt_ns[ss], 36LL * OC * Tp * Bmax);
            // tensor cores: the planes keep the pages side by side in each
            // channel row ([36][C][B*Tp]), so one plane GEMM's rows run over
            // all pages — a 25 x 25 conv's 49 tiles per page fill 128-row M
            // tiles instead of 38 % of one per page.  The SIMT fallback keeps
            // the per-page layout [B*36][C][Tp].
            const bool fold = use_tc && IC % 4 == 0;
            const long long ldt = fold ? (long long)Bmax * Tp : Tp;
            const long long in_ps = IC * ldt, out_ps = OC * ldt;
            const long long bstr_in = fold ? Tp : 36 * in_ps, bstr_out = fold ? Tp : 36 * out_ps;
            push(name + ".wg_in", PPDL_STEP_WG_INPUT, 0.0,
                 4.0 * ((double)IC * x.plane() + 36.0 * IC * T), [=]() {
                return launch_wg4_input(x.p, x.bs, wg_dt_s[ss], IC, x.H, x.W, TW, TH, 1, nb, st,
                                        ldt, in_ps, bstr_in);
            });
            std::shared_ptr<TcGemm> g;
            if (fold) {
                // B = wg4 as K-major TF32 halves [36][OC][IC]; A (the dt planes)
                // exists only once the scratch is allocated -> plan in finalize
                float *bhi = dalloc(36LL * IC * OC), *blo = dalloc(36LL * IC * OC);
                if (!ok) return;
                if (launch_wg4_kmajor_split(wg4, bhi, blo, IC, OC, st) != OK) fail("wg4 split");
                g = std::make_shared<TcGemm>();
                finalizers.push_back([=]() {
                    TcEpilogue e;
                    e.C = wg_yt_s[ss]; e.ldc_m = 1; e.ldc_n = ldt; e.c_bs = out_ps;
                    if (!tc_gemm_plan(g.get(), (int)ldt, OC, IC, 36, wg_dt_s[ss], 1, ldt, in_ps,
                                      bhi, blo, 36, e))
                        g->ok = false;
                });
            }
            push(name + ".wg_madd", PPDL_STEP_WG_MADD, 2.0 * 36 * T * IC * OC,
                 4.0 * (36.0 * T * (IC + OC) + 36.0 * IC * OC), [=]() {
                if (g) return g->ok ? run_tc(g, Tp, 36) : ERR_SHAPE;
                GemmArgs q;
                q.M = OC; q.N = T; q.K = IC; q.batch = nb * 36;
                q.A = {wg4, 1, OC, 36, 0, (long long)IC * OC};
                q.B = {wg_dt_s[ss], Tp, 1, 1, (long long)IC * Tp, 0};
                q.C = wg_yt_s[ss]; q.ldc_m = Tp; q.ldc_n = 1; q.c_bs_hi = (long long)OC * Tp;
                return launch_gemm_simt(q, st);
            });
            push(name + ".wg_out", PPDL_STEP_WG_OUTPUT, 0.0,
                 4.0 * (36.0 * OC * T + (double)OC * OH * OW * (res_mode ? 2 : 1)), [=]() {
                return launch_wg4_output(wg_yt_s[ss], bp, y.p, y.bs, res.p, res.bs, res_mode, OC, OH, OW,
                                         TW, TH, act, nb, st, ldt, out_ps, bstr_out);
            });
            return;
        }
        // the stem's first conv (27 products per output into 32 channels):
        // direct FP32 on the CUDA cores, 157 us against 196 us for the
        // implicit GEMM, whose k-blocks would be two-thirds padding.  The k2
        // stem convs (64 and 128 products) measured faster on the tensor cores
        // (168 / 206 us against 223 / 219 us direct), so the forward keeps them
        // there.
        if (!res_mode && IC * K * K <= 32 && conv_direct_ok(IC, OC, K, s)) {
            push(name, PPDL_STEP_CONV_DIRECT, 2.0 * OC * OH * OW * IC * K * K,
                 4.0 * ((double)IC * x.plane() + (double)OC * OH * OW), [=]() {
                return launch_conv_direct(x.p, x.bs, wp, bp, y.p, y.bs, IC, x.H, x.W, OC, K, s, p,
                                          OH, OW, act, nb, st);
            });
            return;
        }
        // k3-s2 / k2: implicit GEMM on the CHW input (no im2col buffer)
        if (use_tc) {
            auto g = plan_conv_implicit(x, K, s, p, OC, OH, OW, wp,
                                        chw_epilogue(y, bp, act, res, res_mode), name);
            if (g) {
                push(name, PPDL_STEP_GEMM_IMPLICIT, 2.0 * OC * OH * OW * IC * K * K,
                     4.0 * ((double)IC * x.plane() + (double)OC * OH * OW),
                     [=]() { return run_tc(g, 0); });
                return;
            }
        }
        push(name, PPDL_STEP_GEMM_IMPLICIT, 2.0 * OC * OH * OW * IC * K * K,
             4.0 * ((double)IC * x.plane() + (double)OC * OH * OW), [=]() {
            GemmArgs g;
            g.M = OC; g.N = OH * OW; g.K = IC * K * K; g.batch = nb;
            g.A = {wp, (long long)IC * K * K, 1};
            g.B = {x.p, 0, 0, 1, x.bs, 0};
            g.conv = {K, s, p, x.H, x.W, OW};
            g.C = y.p; g.ldc_m = y.plane(); g.ldc_n = 1; g.c_bs_hi = y.bs;
            g.bias = bp; g.bias_mode = 1; g.act = act;
            if (res_mode) {
                g.res = {res.p, res.plane(), 1, 1, res.bs, 0};
                g.res_mode = res_mode;
            }
            return launch_gemm_simt(g, st);
        });
    }

    // 1x1 conv writing token-major rows [row0, row0 + H*W) of a [B][T][256]
    // sequence (decoder input projection + flatten + concat, :786-789)
    void conv1x1_tok(const V &x, const S &y, int row0, const std::string &name) {
        const WT &wt = W(name + ".weight");
        const WT &bt = W(name + ".bias");
        if (!ok) return;
        const int IC = (int)wt.ne[2], OC = (int)wt.ne[3];
        if (wt.ne[0] != 1 || IC != x.C || OC != y.D) {
            fail("conv " + name + ": shape mismatch");
            return;
        }
        const float *wp = wt.p, *bp = bt.p;
        TcEpilogue e;
        e.C = y.p + (long long)row0 * y.D; e.ldc_m = y.D; e.ldc_n = 1; e.c_bs = y.bs();
        e.bias = bp;
        if (use_tc && tc_shape_ok(x.p, x.plane(), x.bs, IC)) {
            const Split wsp = split(wp, (long long)OC * IC);
            auto g = std::make_shared<TcGemm>();
            if (ok && tc_gemm_plan(g.get(), (int)x.plane(), OC, IC, Bmax, x.p, 1, x.plane(), x.bs,
                                   wsp.hi, wsp.lo, 1, e)) {
                push(name, PPDL_STEP_GEMM_1X1, 2.0 * OC * x.plane() * IC,
                     4.0 * ((double)IC + OC) * x.plane(), [=]() { return run_tc(g, 0); });
                return;
            }
        } else if (use_tc) {
            auto g = plan_conv1x1_rows(x, OC, wp, e);
            if (g) {
                push(name, PPDL_STEP_GEMM_1X1, 2.0 * OC * x.plane() * IC,
                     4.0 * ((double)IC + OC) * x.plane(), [=]() { return run_tc(g, 0); });
                return;
            }
        }
        push(name, PPDL_STEP_GEMM_1X1, 2.0 * OC * x.plane() * IC,
             4.0 * ((double)IC + OC) * x.plane(), [=]() {
            GemmArgs g;
            g.M = OC; g.N = (int)x.plane(); g.K = IC; g.batch = nb;
            g.A = {wp, IC, 1};
            g.B = {x.p, x.plane(), 1, 1, x.bs, 0};
            g.C = y.p + (long long)row0 * y.D; g.ldc_m = 1; g.ldc_n = y.D; g.c_bs_hi = y.bs();
            g.bias = bp; g.bias_mode = 1;
            return launch_gemm_simt(g, st);
        });
    }

    // y = act(x W^T + b) (+ res), rows of all pages folded into M
    void lin(const S &x, const S &y, const std::string &name, int act = ACT_NONE,
             const S &res = S(), int max_ctas = 0) {
        lin_cat(x, y, {name}, name, act, res, max_ctas);
    }

    // Linears of one input as one GEMM: their weights stacked row-wise at
    // init ([sum of outs][in], biases likewise), their outputs side by side
    // in y's columns.  Each output element is the same dot product as in
    // the separate linear.
    void lin_cat(const S &x, const S &y, const std::vector<std::string> &names,
                 const std::string &name, int act = ACT_NONE, const S &res = S(),
                 int max_ctas = 0) {
        std::vector<const WT *> ws, bs;
        for (const auto &n : names) {
            ws.push_back(&W(n + ".weight"));
            bs.push_back(&W(n + ".bias"));
        }
        if (!ok) return;
        const int in = (int)ws[0]->ne[0];
        int out = 0;
        for (size_t i = 0; i < ws.size(); i++) {
            if ((int)ws[i]->ne[0] != in || bs[i]->ne[0] != ws[i]->ne[1]) {
                fail("linear " + name + ": stacked weights disagree");
                return;
            }
            out += (int)ws[i]->ne[1];
        }
        if (in != x.D || out != y.D || x.T != y.T) {
            fail("linear " + name + ": shape mismatch");
            return;
        }
        const float *wp = ws[0]->p, *bp = bs[0]->p;
        if (ws.size() > 1) {
            float *wc = dalloc((long long)out * in), *bc = dalloc(out);
            if (!ok) return;
            long long r = 0;
            for (size_t i = 0; i < ws.size(); i++) {
                const long long o = ws[i]->ne[1];
                if (cudaMemcpy(wc + r * in, ws[i]->p, sizeof(float) * o * in,
                               cudaMemcpyDeviceToDevice) != cudaSuccess ||
                    cudaMemcpy(bc + r, bs[i]->p, sizeof(float) * o, cudaMemcpyDeviceToDevice) !=
                        cudaSuccess) {
                    fail("linear " + name + ": weight stacking failed");
                    return;
                }
                r += o;
            }
            wp = wc;
            bp = bc;
        }
        if (use_tc && in % 4 == 0 && ((uintptr_t)x.p & 15) == 0) {
            const Split wsp = split(wp, (long long)out * in);
            TcEpilogue e;
            e.C = y.p; e.ldc_m = out; e.ldc_n = 1;
            e.bias = bp; e.act = act;
            if (res.p) {
                e.res = res.p; e.res_ldm = out; e.res_ldn = 1; e.res_mode = 2;
            }
            auto g = std::make_shared<TcGemm>();
            if (ok && tc_gemm_plan(g.get(), Bmax * x.T, out, in, 1, x.p, 0, in, 0, wsp.hi, wsp.lo, 1,
                                   e)) {
                // a long K (the decoder's 2048 -> 256 linear: 64 k-blocks per
                // tile over 114 tiles) splits into ranges of about 24
                // k-blocks.  The split depends on K only, so every batch
                // capacity sums each output in the same order.
                const int kbl = (in + 31) / 32;
                if (max_ctas == 0 && kbl >= 48) {
                    int sp = (kbl + 23) / 24;
                    if (sp > 8) sp = 8;
                    float *ws = dalloc((long long)sp * Bmax * x.T * out);
                    auto h = std::make_shared<TcGemm>();
                    if (ok && ws &&
                        tc_gemm_plan_split_k(h.get(), Bmax * x.T, out, in, x.p, 0, in, wsp.hi,
                                             wsp.lo, e, sp, ws))
                        g = h;
                }
                g->max_ctas = max_ctas;
                const int T = x.T;
                push(name, PPDL_STEP_GEMM_LINEAR, 2.0 * x.T * out * in,
                     4.0 * ((double)x.T * (in + out) + (double)in * out),
                     [=]() { return run_tc(g, T); });
                return;
            }
        }
        push(name, PPDL_STEP_GEMM_LINEAR, 2.0 * x.T * out * in,
             4.0 * ((double)x.T * (in + out) + (double)in * out), [=]() {
            GemmArgs g;
            g.M = nb * x.T; g.N = out; g.K = in; g.batch = 1;
            g.A = {x.p, in, 1};
            g.B = {wp, 1, in};
            g.C = y.p; g.ldc_m = out; g.ldc_n = 1;
            g.bias = bp; g.bias_mode = 2; g.act = act;
            if (res.p) {
                g.res = {res.p, out, 1};
                g.res_mode = 2;
            }
            return launch_gemm_simt(g, st);
        });
    }

    // y = LN(x (+ r)); with q given also y2 = y + q in the same pass
    void ln(const S &x, const S &y, const std::string &name, const S &r = S(), const S &q = S(),
            const S &y2 = S()) {
        const WT &g = W(name + ".weight");
        const WT &b = W(name + ".bias");
        if (!ok) return;
        const float *gp = g.p, *bp = b.p;
        push(name, PPDL_STEP_GLUE, 0.0, 4.0 * x.T * kDM * (2 + (r.p ? 1 : 0) + (q.p ? 2 : 0)),
             [=]() {
            return launch_layernorm256_add(x.p, r.p, gp, bp, y.p, q.p, y2.p, (long long)nb * x.T,
                                           st);
        });
    }

    void add(const S &a, const S &b, const S &y) {
        push("add", PPDL_STEP_GLUE, 0.0, 12.0 * y.bs(),
             [=]() { return launch_add(a.p, b.p, y.p, (long long)nb * y.bs(), st); });
    }

    void mlp3(const S &x, const S &y, const std::string &pfx) {
        S h1 = seq(x.T, (int)W(pfx + ".0.weight").ne[1]);
        S h2 = seq(x.T, (int)W(pfx + ".1.weight").ne[1]);
        lin(x, h1, pfx + ".0", ACT_RELU);
        lin(h1, h2, pfx + ".1", ACT_RELU);
        lin(h2, y, pfx + ".2");
    }

    // MHA, 8 heads x 32, q/k from qk_in, v from v_in (src/ppdoclayout.cpp:572-587).
    // Called on lane 0 with qk_in and v_in written there; q and k are one
    // GEMM of stacked weights on lane 0, v is projected on lane 2 beside it.
    // A caller that projected v earlier (on lane 2) passes it as v_pre.
    void mha(const S &qk_in, const S &v_in, const S &out, const std::string &pfx,
             const S &v_pre = S()) {
        const int T = qk_in.T;
        S qk = seq(T, 2 * kDM), o = seq(T, kDM);  // q in columns 0..255, k in 256..511
        S v = v_pre.p ? v_pre : seq(T, kDM);
        int e_v = -1;
        if (!v_pre.p) {
            const int e_in = mark();
            on_lane(2);
            after(e_in);
            lin(v_in, v, pfx + ".v");
            e_v = mark();
            on_lane(0);
        } else {
            on_lane(2);
            e_v = mark();  // v_pre is the latest step of lane 2
            on_lane(0);
        }
        lin_cat(qk_in, qk, {pfx + ".q", pfx + ".k"}, pfx + ".qk");
        // softmax(q k^T / sqrt(32)) v in one launch (scores stay on chip)
        after(e_v);
        push(pfx + ".attn", PPDL_STEP_ATTENTION, 4.0 * kNH * T * T * kHD,
             4.0 * 4.0 * T * kDM, [=]() {
            return launch_attention(qk.p, qk.p + kDM, v.p, o.p, T, kNH, 2 * kDM,
                                    (long long)T * 2 * kDM, kDM, (long long)T * kDM,
                                    1.0f / sqrtf((float)kHD), nb, st);
        });
        lin(o, out, pfx + ".o");
    }

    void hg_block(const V &cat, int in_ch, const std::string &pfx, bool light, const V &out,
                  const V &res = V(), int res_mode = 0) {
        const int mid = (int)W(pfx + (light ? ".l0.c1.weight" : ".l0.weight")).ne[3];
        if (!ok) return;
        V cur = cat.slice(0, in_ch);
        V tmp;
        if (light) tmp = tensor(mid, cat.H, cat.W);
        for (int l = 0; l < 6; l++) {
            const std::string lp = pfx + ".l" + std::to_string(l);
            V dst = cat.slice(in_ch + l * mid, mid);
            if (light) {
                conv(cur, tmp, lp + ".c1", 1, 0, ACT_NONE);
                conv(tmp, dst, lp + ".c2", 1, 2, ACT_RELU);
            } else {
                conv(cur, dst, lp, 1, 1, ACT_RELU);
            }
            cur = dst;
        }
        if (cat.C != in_ch + 6 * mid) fail(pfx + ": concat width mismatch");
        V agg0 = tensor(out.C / 2, cat.H, cat.W);
        conv(cat, agg0, pfx + ".agg0", 1, 0, ACT_RELU);
        conv(agg0, out, pfx + ".agg1", 1, 0, ACT_RELU, res, res_mode);
    }

    // RepVGG block (src/ppdoclayout.cpp:656-661): silu(c1(x) + c2(x)), c1 3x3
    // and c2 1x1, run as one 3x3 conv with c2 folded into c1's centre tap
    // (launch_rep_fold, at load); res: added after the SiLU
    void repvgg(const V &x, const V &y, const std::string &pfx, const V &res = V()) {
        const WT &w3 = W(pfx + ".c1.weight"), &b3 = W(pfx + ".c1.bias");
        const WT &w1 = W(pfx + ".c2.weight"), &b1 = W(pfx + ".c2.bias");
        if (!ok) return;
        const int IC = (int)w3.ne[2], OC = (int)w3.ne[3];
        if (w3.ne[0] != 3 || w3.ne[1] != 3 || w1.ne[0] != 1 || w1.ne[1] != 1 ||
            w1.ne[2] != IC || w1.ne[3] != OC || b3.ne[0] != OC || b1.ne[0] != OC) {
            fail("repvgg " + pfx + ": shape mismatch");
            return;
        }
        float *wm = dalloc(9LL * IC * OC), *bm = dalloc(OC);
        if (!ok) return;
        if (launch_rep_fold(w3.p, b3.p, w1.p, b1.p, wm, bm, IC, OC, st) != OK) {
            fail("repvgg " + pfx + ": fold launch failed");
            return;
        }
        WT wmt, bmt;
        wmt.p = wm;
        for (int i = 0; i < 4; i++) wmt.ne[i] = w3.ne[i];
        bmt.p = bm;
        bmt.ne[0] = OC;
        conv(x, y, pfx + ".c1", 1, 1, ACT_SILU, res, res.p ? 2 : 0, -1, &wmt, &bmt);
    }

    // 1x1 convs of the same input stacked along the output channels: one GEMM
    // writing their outputs as consecutive channel slices of y
    void conv_cat(const V &x, const V &y, const std::vector<std::string> &names,
                  const std::string &name, int act) {
        std::vector<const WT *> ws, bs;
        for (const auto &n : names) {
            ws.push_back(&W(n + ".weight"));
            bs.push_back(&W(n + ".bias"));
        }
        if (!ok) return;
        const int64_t IC = ws[0]->ne[2];
        int64_t OC = 0;
        for (size_t i = 0; i < ws.size(); i++) {
            if (ws[i]->ne[0] != 1 || ws[i]->ne[1] != 1 || ws[i]->ne[2] != IC ||
                bs[i]->ne[0] != ws[i]->ne[3]) {
                fail("conv " + name + ": stacked weights disagree");
                return;
            }
            OC += ws[i]->ne[3];
        }
        float *wc = dalloc(OC * IC), *bc = dalloc(OC);
        if (!ok) return;
        long long r = 0;
        for (size_t i = 0; i < ws.size(); i++) {
            const long long o = ws[i]->ne[3];
            if (cudaMemcpy(wc + r * IC, ws[i]->p, sizeof(float) * o * IC,
                           cudaMemcpyDeviceToDevice) != cudaSuccess ||
                cudaMemcpy(bc + r, bs[i]->p, sizeof(float) * o, cudaMemcpyDeviceToDevice) !=
                    cudaSuccess) {
                fail("conv " + name + ": weight stacking failed");
                return;
            }
            r += o;
        }
        WT wt, bt;
        wt.p = wc;
        wt.ne[2] = IC;
        wt.ne[3] = OC;
        bt.p = bc;
        bt.ne[0] = OC;
        conv(x, y, name, 1, 0, act, V(), 0, -1, &wt, &bt);
    }

    // CSP block (src/ppdoclayout.cpp:663-668): c1 and c2 (1x1 + SiLU of x)
    // as one GEMM into [a | c2(x)], three RepVGG blocks on a, the last one
    // adding c2(x) after its SiLU (the reference's final add)
    void csp(const V &x, const V &out, const std::string &pfx) {
        V ab = tensor(512, x.H, x.W), t1 = tensor(256, x.H, x.W), t2 = tensor(256, x.H, x.W);
        const V a = ab.slice(0, 256), c2o = ab.slice(256, 256);
        conv_cat(x, ab, {pfx + ".c1", pfx + ".c2"}, pfx + ".c1c2", ACT_SILU);
        repvgg(a, t1, pfx + ".bn0");
        repvgg(t1, t2, pfx + ".bn1");
        repvgg(t2, out, pfx + ".bn2", c2o);
    }

    void interp(const V &x, const V &y, bool bilinear, const V &base = V()) {
        push("interp", PPDL_STEP_GLUE, 0.0,
             4.0 * ((double)x.C * x.plane() + (double)y.C * y.plane() * (base.p ? 2 : 1)), [=]() {
            return launch_interp(x.p, x.bs, y.p, y.bs, base.p, base.bs, x.C, x.H, x.W, y.H, y.W,
                                 bilinear, nb, st);
        });
    }

    // ---- the network (src/ppdoclayout.cpp:598-882) ---------------------------
    void build() {
        img = tensor(3, kImg, kImg);
        int32_t *ohw = nullptr;
        if (cudaMalloc(&ohw, sizeof(int32_t) * 2 * Bmax) != cudaSuccess) fail("cudaMalloc");
        allocs.push_back(ohw);
        ori_hw = ohw;

        // stem (:618-631)
        V x1 = tensor(32, 400, 400);
        conv(img, x1, "stem1", 2, 1, ACT_RELU);
        dump_chw("stem1", x1);
        V a1 = tensor(16, 400, 400);
        conv(x1, a1, "stem2a", 1, 0, ACT_RELU, V(), 0, 1);
        V scat = tensor(64, 400, 400);  // concat(pool, stem2b)
        conv(a1, scat.slice(32, 32), "stem2b", 1, 0, ACT_RELU, V(), 0, 1);
        {
            V xs = x1, ys = scat.slice(0, 32);
            push("stem.pool", PPDL_STEP_GLUE, 0.0, 8.0 * xs.C * xs.plane(), [=]() {
                return launch_maxpool2_pad(xs.p, xs.bs, ys.p, ys.bs, xs.C, xs.H, xs.W, nb, st);
            });
        }
        V x3 = tensor(32, 200, 200);
        conv(scat, x3, "stem3", 2, 1, ACT_RELU);
        // stage 0: stem4 writes the first slice of the HG-block concat
        V c0 = tensor(48 + 6 * 48, 200, 200);
        conv(x3, c0.slice(0, 48), "stem4", 1, 0, ACT_RELU);
        dump_chw("stem", c0.slice(0, 48));
        V s0 = tensor(128, 200, 200);
        hg_block(c0, 48, "st0.b0", false, s0);
        dump_chw("st0", s0);
        // stage 1
        V c1 = tensor(128 + 6 * 96, 100, 100);
        conv(s0, c1.slice(0, 128), "st1.ds", 2, 1, ACT_NONE);
        V s1 = tensor(512, 100, 100);
        hg_block(c1, 128, "st1.b0", false, s1);
        dump_chw("st1", s1);
        // stage 2: three light blocks, residual on b1/b2
        V c2a = tensor(512 + 6 * 192, 50, 50);
        conv(s1, c2a.slice(0, 512), "st2.ds", 2, 1, ACT_NONE);
        V c2b = tensor(1024 + 6 * 192, 50, 50);
        hg_block(c2a, 512, "st2.b0", true, c2b.slice(0, 1024));
        V c2c = tensor(1024 + 6 * 192, 50, 50);
        hg_block(c2b, 1024, "st2.b1", true, c2c.slice(0, 1024), c2b.slice(0, 1024), 2);
        V s2 = tensor(1024, 50, 50);
        hg_block(c2c, 1024, "st2.b2", true, s2, c2c.slice(0, 1024), 2);
        dump_chw("st2", s2);
        // stage 3
        V c3 = tensor(1024 + 6 * 384, 25, 25);
        conv(s2, c3.slice(0, 1024), "st3.ds", 2, 1, ACT_NONE);
        V s3 = tensor(2048, 25, 25);
        hg_block(c3, 1024, "st3.b0", true, s3);
        dump_chw("st3", s3);

        // ---- hybrid encoder (:674-729)
        V fcat1 = tensor(512, 100, 100), fcat0 = tensor(512, 50, 50);
        V pcat0 = tensor(512, 50, 50), pcat1 = tensor(512, 25, 25);
        conv(s1, fcat1.slice(256, 256), "enc_in0", 1, 0, ACT_NONE);
        conv(s2, fcat0.slice(256, 256), "enc_in1", 1, 0, ACT_NONE);
        V p32 = tensor(256, 25, 25);
        conv(s3, p32, "enc_in2", 1, 0, ACT_NONE);
        // AIFI (post-norm) on the 625 tokens of p32
        S sq = seq(625, kDM), qk = seq(625, kDM), at = seq(625, kDM), sa1 = seq(625, kDM);
        S f1 = seq(625, (int)W("aifi.fc1.weight").ne[1]), f2 = seq(625, kDM), sa2 = seq(625, kDM);
        push("aifi.to_seq", PPDL_STEP_GLUE, 0.0, 8.0 * 625 * kDM, [=]() {  // [256][625] -> [625][256]
            return launch_transpose(p32.p, p32.bs, sq.p, sq.bs(), kDM, 625, 625, kDM, nb, st);
        });
        {
            S q2 = qk;
            const float *pp = pos;
            push("aifi.pos", PPDL_STEP_GLUE, 0.0, 12.0 * 625 * kDM, [=]() {  // qk = s + pos
                return launch_add_bcast(sq.p, pp, q2.p, sq.bs(), nb, st);
            });
        }
        mha(qk, sq, at, "aifi");
        ln(sq, sa1, "aifi.ln1", at);
        lin(sa1, f1, "aifi.fc1", ACT_GELU);
        lin(f1, f2, "aifi.fc2");
        ln(sa1, sa2, "aifi.ln2", f2);
        V p32a = tensor(256, 25, 25);
        push("aifi.to_chw", PPDL_STEP_GLUE, 0.0, 8.0 * 625 * kDM, [=]() {  // back to CHW
            return launch_transpose(sa2.p, sa2.bs(), p32a.p, p32a.bs, 625, kDM, kDM, 625, nb, st);
        });
        dump_chw("aifi", p32a);
        // FPN (top-down)
        V lat0 = pcat1.slice(256, 256);
        conv(p32a, lat0, "lat0", 1, 0, ACT_SILU);
        interp(lat0, fcat0.slice(0, 256), false);
        V f16 = tensor(256, 50, 50);
        csp(fcat0, f16, "fpn0");
        V lat1 = pcat0.slice(256, 256);
        conv(f16, lat1, "lat1", 1, 0, ACT_SILU);
        interp(lat1, fcat1.slice(0, 256), false);
        V f8 = tensor(256, 100, 100);
        csp(fcat1, f8, "fpn1");
        dump_chw("f8", f8);
        const int e_f8 = mark();
        // PAN (bottom-up)
        conv(f8, pcat0.slice(0, 256), "pand0", 2, 1, ACT_SILU);
        V n16 = tensor(256, 50, 50);
        csp(pcat0, n16, "pan0");
        dump_chw("n16", n16);
        const int e_n16 = mark();
        conv(n16, pcat1.slice(0, 256), "pand1", 2, 1, ACT_SILU);
        V n32 = tensor(256, 25, 25);
        csp(pcat1, n32, "pan1");
        dump_chw("n32", n32);
        // mask feature head, on lane 2 with its own scratch set: each level
        // starts once its feature exists (f8 after the FPN, n16 and n32 along
        // the PAN), overlapping the PAN, the decoder input, the encoder head
        // and the top-300 selection until the encoder's mask GEMM needs it
        const int e_n32 = mark();
        on_lane(2);
        after(e_f8);
        scratch = 1;
        V hs = tensor(64, 100, 100);
        conv(f8, hs, "mh0.0", 1, 1, ACT_SILU);
        V h1 = tensor(64, 50, 50);
        after(e_n16);
        conv(n16, h1, "mh1.0", 1, 1, ACT_SILU);
        interp(h1, hs, true, hs);  // h0 + up(h1)
        V h2 = tensor(64, 25, 25), h2i = tensor(64, 50, 50), h2b = tensor(64, 50, 50);
        after(e_n32);
        conv(n32, h2, "mh2.0", 1, 1, ACT_SILU);
        interp(h2, h2i, true);
        conv(h2i, h2b, "mh2.2", 1, 1, ACT_SILU);
        interp(h2b, hs, true, hs);  // (h0 + h1) + up(h2)
        V mo = tensor(64, 100, 100), moi = tensor(64, 200, 200), ml = tensor(64, 200, 200);
        conv(hs, mo, "mh.out", 1, 1, ACT_SILU);
        interp(mo, moi, true);
        conv(s0, ml, "mlat", 1, 1, ACT_SILU, moi, 2);  // up(mf) + mlat(x4)
        V mb = tensor(64, 200, 200), mfeat = tensor(32, 200, 200);
        conv(ml, mb, "mout.base", 1, 1, ACT_SILU);
        conv(mb, mfeat, "mout.conv", 1, 0, ACT_NONE);
        dump_chw("mask_feat", mfeat);
        scratch = 0;
        const int e_mf = mark();
        on_lane(0);

        // ---- decoder input, two-stage selection (:781-821)
        S source = seq(kNTok, kDM);
        conv1x1_tok(f8, source, 0, "dec_in0");
        conv1x1_tok(n16, source, 10000, "dec_in1");
        conv1x1_tok(n32, source, 12500, "dec_in2");
        dump_seq("source", source);
        // the six layers' value projections of `source` (:836) as one GEMM
        // of stacked weights, 13125*B x 1536 x 256, on lane 1 beside the
        // encoder head, on at most kVpCtas SMs so that the chain keeps the
        // rest; layer i's MSDA reads columns 256i .. 256i + 255 of each row
        S values_all = seq(kNTok, 6 * kDM);
        int e_vp_all;
        {
            const int e_src = mark();
            on_lane(1);
            after(e_src);
            std::vector<std::string> vps;
            for (int i = 0; i < 6; i++) vps.push_back("dec" + std::to_string(i) + ".ca.vp");
            lin_cat(source, values_all, vps, "dec.ca.vp", ACT_NONE, S(), kVpCtas);
            e_vp_all = mark();
            on_lane(0);
        }
        S memory = seq(kNTok, kDM), eo = seq(kNTok, kDM), om = seq(kNTok, kDM);
        S ecls = seq(kNTok, kNC);
        {
            const float *vp = valid;
            push("memory", PPDL_STEP_GLUE, 0.0, 8.0 * kNTok * kDM, [=]() {
                return launch_row_scale(source.p, vp, memory.p, kNTok, kDM, nb, st);
            });
        }
        lin(memory, eo, "enc_out.l");
        ln(eo, om, "enc_out.ln");
        lin(om, ecls, "score_head");
        int32_t *topk = nullptr;
        if (cudaMalloc(&topk, sizeof(int32_t) * kNQ * Bmax) != cudaSuccess) fail("cudaMalloc");
        allocs.push_back(topk);
        enc_topk = topk;
        push("topk300", PPDL_STEP_TOPK, 0.0, 4.0 * kNTok * kNC,
             [=]() { return launch_topk(ecls.p, topk, kNTok, kNC, kNQ, nb, st); });
        if (dumps) dump_list.push_back({"topk_idx", topk, {kNQ, 1, 1, 1}, "i32", kNQ * 4});
        S target = seq(kNQ, kDM);
        push("target", PPDL_STEP_GLUE, 0.0, 8.0 * kNQ * kDM, [=]() {
            return launch_gather_rows(om.p, topk, target.p, kNTok, kNQ, kDM, nb, st);
        });
        dump_seq("target", target);
        S tq = seq(kNQ, kDM), mq0 = seq(kNQ, 32);
        ln(target, tq, "dec_norm");
        mlp3(tq, mq0, "mq");
        const V mf = mfeat;
        // mask logits [b][q][p] = sum_c mq[b][q][c] mf[b][c][p], thresholded
        // (> 0) and packed 1 bit per pixel in the GEMM's epilogue — every
        // consumer (mask -> box, the result masks) needs only the threshold.
        // On the tensor cores A = mf (pixels x 32 channels, M-major) and
        // B = mq, split into TF32 halves per forward (it is an activation).
        uint32_t *encm = nullptr;
        if (cudaMalloc(&encm, sizeof(uint32_t) * (size_t)kNQ * kMaskWords * Bmax) != cudaSuccess)
            fail("cudaMalloc");
        allocs.push_back(encm);
        float *mq_hi = dalloc((long long)kNQ * 32 * Bmax), *mq_lo = dalloc((long long)kNQ * 32 * Bmax);
        float *mask_f32 = nullptr;  // float logits, only for the SIMT fallback
        auto mask_gemm = [&, mf, mq_hi, mq_lo](const S &mq, uint32_t *dst) {
            if (use_tc && tc_shape_ok(mf.p, mf.plane(), mf.bs, 32)) {
                TcEpilogue e;
                e.C = reinterpret_cast<float *>(dst);
                e.ldc_m = 1; e.ldc_n = kMaskPix; e.c_bs = (long long)kNQ * kMaskPix;
                auto g = std::make_shared<TcGemm>();
                if (ok && tc_gemm_plan(g.get(), kMaskPix, kNQ, 32, Bmax, mf.p, 1, mf.plane(), mf.bs,
                                       mq_hi, mq_lo, Bmax, e) &&
                    tc_gemm_set_bits_output(g.get(), dst, kMaskWords,
                                            (long long)kNQ * kMaskWords)) {
                    push("mask_gemm", PPDL_STEP_GEMM_LINEAR, 2.0 * kNQ * kMaskPix * 32,
                         4.0 * ((double)kNQ * kMaskWords + 32.0 * kMaskPix), [=]() {
                        TRY(launch_tf32_split(mq.p, mq_hi, mq_lo, (long long)nb * mq.bs(), st));
                        return run_tc(g, 0);
                    });
                    return;
                }
            }
            if (!mask_f32) mask_f32 = dalloc((long long)kNQ * kMaskPix * Bmax);
            float *mf32 = mask_f32;
            push("mask_gemm", PPDL_STEP_GEMM_LINEAR, 2.0 * kNQ * kMaskPix * 32,
                 4.0 * ((double)kNQ * kMaskPix + 32.0 * kMaskPix), [=]() {
                GemmArgs g;
                g.M = kNQ; g.N = kMaskPix; g.K = 32; g.batch = nb;
                g.A = {mq.p, 32, 1, 1, mq.bs(), 0};
                g.B = {mf.p, mf.plane(), 1, 1, mf.bs, 0};
                g.C = mf32; g.ldc_m = kMaskPix; g.ldc_n = 1; g.c_bs_hi = (long long)kNQ * kMaskPix;
                TRY(launch_gemm_simt(g, st));
                return launch_pack_mask_bits(mf32, dst, nb, st);
            });
        };
        after(e_mf);
        mask_gemm(mq0, encm);
        if (dumps)
            dump_list.push_back({"enc_mask_bits", encm, {kMaskWords, kNQ, 1, 1}, "u32",
                                 (size_t)kNQ * kMaskWords * 4});
        S refu = seq(kNQ, 4), ref = seq(kNQ, 4);
        push("mask_box", PPDL_STEP_MASKBOX, 0.0, 4.0 * kNQ * kMaskWords,
             [=]() { return launch_mask_box_bits(encm, refu.p, nb * kNQ, st); });
        dump_seq("init_ref_unact", refu);
        push("ref", PPDL_STEP_GLUE, 0.0, 8.0 * refu.bs(),
             [=]() { return launch_sigmoid(refu.p, ref.p, (long long)nb * refu.bs(), st); });

        // ---- decoder layers (:824-851)
        // lane 2 takes the self-attention's v projection off the chain (from
        // x, beside the previous layer's box head and this layer's query
        // position MLP)
        // The box head's last linear, the refinement of ref and the next
        // layer's first query-position linear run as one launch
        // (launch_box_refine); layer 0's query-position input comes from the
        // encoder's boxes.
        const WT &bw0 = W("bbox_head.0.weight"), &bw1 = W("bbox_head.1.weight");
        const WT &bw2 = W("bbox_head.2.weight"), &bb2 = W("bbox_head.2.bias");
        const WT &qw0 = W("qpos.0.weight"), &qb0 = W("qpos.0.bias");
        if (!ok) return;
        const int nqp = (int)qw0.ne[1];
        if (bw2.ne[0] != 256 || bw2.ne[1] != 4 || qw0.ne[0] != 4 || bw0.ne[1] != bw1.ne[0])
            fail("box head / query-position shapes");
        S x = target;
        int e_x = mark();
        S qp1 = seq(kNQ, nqp);
        lin(ref, qp1, "qpos.0", ACT_RELU);
        for (int i = 0; i < 6; i++) {
            const std::string dp = "dec" + std::to_string(i);
            const float *value_p = values_all.p + (long long)i * kDM;
            S v = seq(kNQ, kDM);
            on_lane(2);
            after(e_x);
            // at most 34 CTAs: the chain's 2400-row GEMMs beside it take 114
            // (19 row tiles x 6 column tiles), so neither waits for SMs
            lin(x, v, dp + ".sa.v", ACT_NONE, S(), 34);
            on_lane(0);
            S qpos = seq(kNQ, kDM);
            lin(qp1, qpos, "qpos.1");
            S qk2 = seq(kNQ, kDM), sa = seq(kNQ, kDM), x1 = seq(kNQ, kDM);
            add(x, qpos, qk2);
            mha(qk2, x, sa, dp + ".sa", v);
            // sampling offsets (columns 0..191) and attention logits (192..287)
            S z = seq(kNQ, kDM), sa_lg = seq(kNQ, 288), ca = seq(kNQ, kDM);
            ln(x, x1, dp + ".ln1", sa, qpos, z);  // x1 and z = x1 + qpos
            lin_cat(z, sa_lg, {dp + ".ca.so", dp + ".ca.aw"}, dp + ".ca.so_aw");
            if (i == 0) after(e_vp_all);
            push(dp + ".msda", PPDL_STEP_MSDA, 0.0,
                 4.0 * ((double)kNTok * kDM + kNQ * (192.0 + 96.0 + 4.0 + kDM)), [=]() {
                return launch_msda(value_p, sa_lg.p, sa_lg.p + 192, ref.p, ca.p, kNQ, nb, false,
                                   288, 288, st, 6 * kDM);
            });
            S cao = seq(kNQ, kDM), x2 = seq(kNQ, kDM);
            lin(ca, cao, dp + ".ca.op");
            ln(x1, x2, dp + ".ln2", cao);
            S fa = seq(kNQ, (int)W(dp + ".fc1.weight").ne[1]), fb = seq(kNQ, kDM),
              x3 = seq(kNQ, kDM);
            lin(x2, fa, dp + ".fc1", ACT_RELU);
            lin(fa, fb, dp + ".fc2");
            ln(x2, x3, dp + ".ln3", fb);
            static const char *hn[6] = {"hidden0", "hidden1", "hidden2",
                                        "hidden3", "hidden4", "hidden5"};
            dump_seq(hn[i], x3);
            e_x = mark();
            S bh1 = seq(kNQ, (int)bw0.ne[1]), bh2 = seq(kNQ, (int)bw1.ne[1]);
            lin(x3, bh1, "bbox_head.0", ACT_RELU);
            lin(bh1, bh2, "bbox_head.1", ACT_RELU);
            const S qpn = i < 5 ? seq(kNQ, nqp) : S();
            {
                const float *w2 = bw2.p, *b2 = bb2.p, *wq = qw0.p, *bq = qb0.p;
                push(dp + ".box_refine", PPDL_STEP_GLUE, 2.0 * kNQ * (4 * 256 + 4.0 * nqp),
                     4.0 * kNQ * (256 + 8 + (qpn.p ? nqp : 0)), [=]() {
                    return launch_box_refine(bh2.p, w2, b2, ref.p, wq, bq, qpn.p, nb * kNQ, nqp,
                                             st);
                });
            }
            qp1 = qpn;
            x = x3;
        }

        // ---- heads (:853-866)
        S outq = seq(kNQ, kDM), mq6 = seq(kNQ, 32);
        logits = seq(kNQ, kNC);
        boxes = ref;
        ln(x, outq, "dec_norm");
        lin(outq, logits, "score_head");
        mlp3(outq, mq6, "mq");
        uint32_t *mask_bits_q = nullptr;  // packed masks of the 300 queries
        if (cudaMalloc(&mask_bits_q, sizeof(uint32_t) * (size_t)kNQ * kMaskWords * Bmax) !=
            cudaSuccess)
            fail("cudaMalloc");
        allocs.push_back(mask_bits_q);
        mask_gemm(mq6, mask_bits_q);
        // the reading-order head on lane 2, beside the class/mask heads
        S oh = seq(kNQ, kDM), gp = seq(kNQ, 128);
        on_lane(2);
        after(e_x);
        lin(x, oh, "order5");
        lin(oh, gp, "gp");
        order = seq(kNQ, kNQ);
        {
            const S o = order;
            push("order", PPDL_STEP_ATTENTION, 2.0 * kNQ * kNQ * 64, 4.0 * kNQ * (kNQ + 128.0),
                 [=]() {  // order[b][i][j] = q_i . k_j / 8
                GemmArgs g;
                g.M = kNQ; g.N = kNQ; g.K = 64; g.batch = nb;
                g.A = {gp.p, 128, 1, 1, gp.bs(), 0};
                g.B = {gp.p + 64, 1, 128, 1, gp.bs(), 0};
                g.C = o.p; g.ldc_m = kNQ; g.ldc_n = 1; g.c_bs_hi = o.bs();
                g.alpha = 0.125f;
                return launch_gemm_simt(g, st);
            });
        }
        const int e_order = mark();
        on_lane(0);
        // ---- postprocess (:927-993)
        dets = dalloc((long long)kNQ * 7 * Bmax);
        if (cudaMalloc(&sel, sizeof(int32_t) * kNQ * Bmax) != cudaSuccess) fail("cudaMalloc");
        allocs.push_back(sel);
        if (cudaMalloc(&rank, sizeof(int32_t) * kNQ * Bmax) != cudaSuccess) fail("cudaMalloc");
        allocs.push_back(rank);
        if (cudaMalloc(&masks, sizeof(int32_t) * (size_t)kNQ * kMaskPix * Bmax) != cudaSuccess)
            fail("cudaMalloc");
        allocs.push_back(masks);
        if (cudaMalloc(&mask_bits, sizeof(uint32_t) * (size_t)kNQ * kMaskWords * Bmax) !=
            cudaSuccess)
            fail("cudaMalloc");
        allocs.push_back(mask_bits);
        {
            // the forward's mask output is packed (1 bit per pixel); the
            // int32 form of the reference's result is expanded from it only
            // for the calls that return it (expand_masks)
            const S lg = logits, bx = boxes, od = order;
            uint32_t *mb = mask_bits;
            after(e_order);
            push("postprocess", PPDL_STEP_POSTPROCESS, 0.0,
                 4.0 * ((double)kNQ * kNQ + 2.0 * kNQ * kMaskWords), [=]() {
                return launch_postprocess(lg.p, bx.p, od.p, nullptr, mask_bits_q, ori_hw, rank,
                                          dets, sel, nullptr, mb, nb, st);
            });
        }
        if (!ok) return;
        for (int k = 0; k < 2; k++) {
            wg_dt_s[k] = dalloc(wg_dt_ns[k]);
            wg_yt_s[k] = dalloc(wg_yt_ns[k]);
        }
        if (!ok) return;
        for (auto &f : finalizers) f();
    }

    float *pos = nullptr, *valid = nullptr;

    bool init(const char *path, int device, int max_batch, bool want_dumps) {
        if (device >= 0 && cudaSetDevice(device) != cudaSuccess) {
            fail("cudaSetDevice failed");
            return false;
        }
        cudaGetDevice(&dev);
        Bmax = max_batch;
        nb = max_batch;
        dumps = want_dumps;
        const char *tc_env = getenv("PPDL_TC");
        use_tc = !(tc_env && tc_env[0] == '0');
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
            fail("no CUDA device / stream");
            return false;
        }
        lanes[0] = st;
        for (int l = 1; l < kLanes; l++)
            if (cudaStreamCreateWithFlags(&lanes[l], cudaStreamNonBlocking) != cudaSuccess) {
                fail("stream creation failed");
                return false;
            }
        if (!load(path)) return false;
        // host constants (src/ppdoclayout.cpp:887-923), float64 math as there
        std::vector<float> hp((size_t)kDM * 625), hv(kNTok);
        double omega[64];
        for (int i = 0; i < 64; i++) omega[i] = 1.0 / std::pow(10000.0, (double)i / 64.0);
        for (int h = 0; h < 25; h++)
            for (int x = 0; x < 25; x++) {
                float *p = hp.data() + (size_t)(h * 25 + x) * kDM;
                for (int i = 0; i < 64; i++) {
                    p[i] = (float)std::sin(h * omega[i]);
                    p[64 + i] = (float)std::cos(h * omega[i]);
                    p[128 + i] = (float)std::sin(x * omega[i]);
                    p[192 + i] = (float)std::cos(x * omega[i]);
                }
            }
        static const int LW[3] = {100, 50, 25};
        int t = 0;
        for (int l = 0; l < 3; l++) {
            const float wh = 0.05f * (float)std::pow(2.0f, (float)l);
            for (int y = 0; y < LW[l]; y++)
                for (int x = 0; x < LW[l]; x++) {
                    const float cx = ((float)x + 0.5f) / (float)LW[l];
                    const float cy = ((float)y + 0.5f) / (float)LW[l];
                    const float eps = 1e-2f;
                    const bool okk = cx > eps && cx < 1.0f - eps && cy > eps && cy < 1.0f - eps &&
                                     wh > eps && wh < 1.0f - eps;
                    hv[t++] = okk ? 1.0f : 0.0f;
                }
        }
        pos = dalloc((long long)hp.size());
        valid = dalloc((long long)hv.size());
        if (!ok) return false;
        cudaMemcpy(pos, hp.data(), hp.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(valid, hv.data(), hv.size() * 4, cudaMemcpyHostToDevice);
        build();
        if (!ok) return false;
        if (lane != 0 || !pending.empty()) {
            fail("plan ends off lane 0 or with pending waits");
            return false;
        }
        events.resize(n_events + kLanes);
        for (auto &e : events)
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
                e = nullptr;
                fail("event creation failed");
                return false;
            }
        if (cudaStreamSynchronize(st) != cudaSuccess) {
            fail("weight transform failed");
            return false;
        }
        return true;
    }

    // Enqueues the plan on its lanes: every side lane first waits for the
    // work already on lane 0 (fork) and lane 0 ends by waiting for every side
    // lane (join), so the forward is ordered on the context's stream as one
    // unit, eager or captured.  The launch closures read `st` when called, so
    // it names the step's lane while the step is enqueued.
    Status exec(const std::function<bool(int)> &after_step = nullptr) {
        cudaStream_t main = lanes[0];
        const int fork = n_events, join = n_events + 1;
        if (cudaEventRecord(events[fork], main) != cudaSuccess) return ERR_CUDA;
        for (int l = 1; l < kLanes; l++)
            if (cudaStreamWaitEvent(lanes[l], events[fork], 0) != cudaSuccess) return ERR_CUDA;
        Status s = OK;
        for (size_t i = 0; i < plan.size(); i++) {
            const Step &f = plan[i];
            st = lanes[f.lane];
            for (int e : f.waits)
                if (cudaStreamWaitEvent(st, events[e], 0) != cudaSuccess) s = ERR_CUDA;
            if (s == OK) s = f.fn();
            if (s == OK && after_step && !after_step((int)i)) s = ERR_CUDA;
            if (s == OK && f.record >= 0 && cudaEventRecord(events[f.record], st) != cudaSuccess)
                s = ERR_CUDA;
            if (s != OK) break;
        }
        st = main;
        for (int l = 1; l < kLanes; l++) {  // join even after an error (ends a capture cleanly)
            const int e = join + l - 1;
            if (cudaEventRecord(events[e], lanes[l]) != cudaSuccess ||
                cudaStreamWaitEvent(main, events[e], 0) != cudaSuccess)
                s = s == OK ? ERR_CUDA : s;
        }
        return s;
    }

    // int32 masks of the last n pages from the packed ones (the reference's
    // result format, 48 MB per page)
    Status expand_masks(int n) {
        return launch_unpack_mask_bits(mask_bits, masks, (long long)n * kNQ, st);
    }

    // Runs the plan for n pages: eagerly the first time (sets kernel
    // attributes), then from a captured CUDA graph per batch size.
    Status run(int n) {
        nb = n;
        auto it = graphs.find(n);
        if (it != graphs.end()) {
            return cudaGraphLaunch(it->second, st) == cudaSuccess ? OK : ERR_CUDA;
        }
        TRY(exec());
        if (cudaStreamSynchronize(st) != cudaSuccess) return ERR_CUDA;
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
            return OK;  // eager result stands; no graph
        const Status s = exec();
        if (cudaStreamEndCapture(st, &g) != cudaSuccess || s != OK) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            return s;
        }
        cudaGraphExec_t ge = nullptr;
        if (cudaGraphInstantiate(&ge, g, 0) == cudaSuccess) graphs[n] = ge;
        cudaGraphDestroy(g);
        return OK;
    }
};

}  // namespace ppdl

// ============================================================ C ABI ========
// Two-deep pipeline of ppdl_submit_batch / ppdl_wait_batch: slot s = ticket
// % 2 owns a device staging buffer for the pages (filled on the copy-in
// stream, copied into the forward's input on the compute stream), device
// and pinned host copies of the dets and packed masks (copied out on the
// copy-out stream), and the events that order the three streams.
struct PpdlPipe {
    bool ready = false;
    cudaStream_t h2d = nullptr, d2h = nullptr;
    float *d_in[2] = {}, *d_dets[2] = {};
    int32_t *d_hw[2] = {};
    uint32_t *d_bits[2] = {};
    float *h_dets[2] = {};
    uint32_t *h_bits[2] = {};
    cudaEvent_t in_ready[2] = {}, in_free[2] = {}, out_ready[2] = {}, out_done[2] = {},
                t0[2] = {}, t1[2] = {};
    long long ticket_of[2] = {-1, -1}, next = 0;
    int n_of[2] = {0, 0};
};

struct ppdl_ctx {
    std::unique_ptr<ppdl::Model> m;
    float *h_dets = nullptr;
    int32_t *h_masks = nullptr;
    bool computed = false;
    int last_n = 0;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    PpdlPipe pipe;
};

namespace {

void pipe_release(PpdlPipe &p) {
    if (p.h2d) cudaStreamSynchronize(p.h2d);
    if (p.d2h) cudaStreamSynchronize(p.d2h);
    for (int s = 0; s < 2; s++) {
        if (p.d_in[s]) cudaFree(p.d_in[s]);
        if (p.d_dets[s]) cudaFree(p.d_dets[s]);
        if (p.d_hw[s]) cudaFree(p.d_hw[s]);
        if (p.d_bits[s]) cudaFree(p.d_bits[s]);
        if (p.h_dets[s]) cudaFreeHost(p.h_dets[s]);
        if (p.h_bits[s]) cudaFreeHost(p.h_bits[s]);
        for (cudaEvent_t e : {p.in_ready[s], p.in_free[s], p.out_ready[s], p.out_done[s], p.t0[s],
                              p.t1[s]})
            if (e) cudaEventDestroy(e);
    }
    if (p.h2d) cudaStreamDestroy(p.h2d);
    if (p.d2h) cudaStreamDestroy(p.d2h);
    p = PpdlPipe();
}

void ctx_release(ppdl_ctx *c) {
    if (!c) return;
    if (c->m) cudaSetDevice(c->m->dev);
    if (c->m) cudaStreamSynchronize(c->m->st);
    pipe_release(c->pipe);
    if (c->h_dets) cudaFreeHost(c->h_dets);
    if (c->h_masks) cudaFreeHost(c->h_masks);
    if (c->e0) cudaEventDestroy(c->e0);
    if (c->e1) cudaEventDestroy(c->e1);
    c->m.reset();
    delete c;
}

bool write_file(const std::string &path, const void *src, size_t n) {
    FILE *f = fopen(path.c_str(), "wb");
    if (!f) return false;
    const size_t wr = fwrite(src, 1, n, f);
    fclose(f);
    return wr == n;
}

int enqueue(ppdl_ctx *c, const float *images, bool images_on_device, int n, const int32_t *ori_hw,
            bool int32_masks = true) {
    ppdl::Model &m = *c->m;
    cudaSetDevice(m.dev);
    const size_t img_bytes = (size_t)3 * ppdl::kImg * ppdl::kImg * sizeof(float);
    if (cudaMemcpyAsync(m.img.p, images, img_bytes * n,
                        images_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                        m.st) != cudaSuccess)
        return 2;
    if (cudaMemcpyAsync(m.ori_hw, ori_hw, sizeof(int32_t) * 2 * n, cudaMemcpyHostToDevice, m.st) !=
        cudaSuccess)
        return 2;
    cudaEventRecord(c->e0, m.st);
    if (m.run(n) != ppdl::OK) {
        fprintf(stderr, "ppdl: forward launch failed: %s\n", cudaGetErrorString(cudaGetLastError()));
        return 2;
    }
    cudaEventRecord(c->e1, m.st);
    if (int32_masks && m.expand_masks(n) != ppdl::OK) return 2;
    c->last_n = n;
    return 0;
}

ppdl_ctx *init_common(const char *path, int backend, int device, int max_batch, int dumps) {
    if (!path) {
        fprintf(stderr, "ppdl: null model path\n");
        return nullptr;
    }
    if (backend != PPDL_BACKEND_CUDA) {
        fprintf(stderr, "ppdl: this build provides the CUDA (B200) backend only\n");
        return nullptr;
    }
    if (max_batch < 1 || max_batch > 64) {
        fprintf(stderr, "ppdl: max_batch must be in 1..64\n");
        return nullptr;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        fprintf(stderr, "ppdl: no GPU backend available\n");
        return nullptr;
    }
    ppdl_ctx *c = new ppdl_ctx();
    c->m.reset(new ppdl::Model());
    if (!c->m->init(path, device, max_batch, dumps != 0)) {
        fprintf(stderr, "ppdl: failed to load %s: %s\n", path, c->m->err.c_str());
        ctx_release(c);
        return nullptr;
    }
    if (cudaHostAlloc(&c->h_dets, sizeof(float) * ppdl::kNQ * 7 * max_batch, 0) != cudaSuccess ||
        cudaHostAlloc(&c->h_masks, sizeof(int32_t) * (size_t)ppdl::kNQ * ppdl::kMaskPix * max_batch,
                      0) != cudaSuccess ||
        cudaEventCreate(&c->e0) != cudaSuccess || cudaEventCreate(&c->e1) != cudaSuccess) {
        fprintf(stderr, "ppdl: host buffer allocation failed\n");
        ctx_release(c);
        return nullptr;
    }
    fprintf(stderr, "ppdl: loaded %s (%zu tensors) on device %d, batch capacity %d, %zu launches\n",
            path, c->m->w.size(), c->m->dev, max_batch, c->m->plan.size());
    return c;
}

}  // namespace

extern "C" {

PPDL_API ppdl_ctx *ppdl_init_dev(const char *model_path, int backend, int device, int max_batch,
                                 int enable_dumps) {
    return init_common(model_path, backend, device, max_batch, enable_dumps);
}

PPDL_API ppdl_ctx *ppdl_init_ex(const char *model_path, int backend, int enable_dumps) {
    return init_common(model_path, backend, -1, 1, enable_dumps);
}

PPDL_API ppdl_ctx *ppdl_init(const char *model_path, int backend) {
    return init_common(model_path, backend, -1, 1, 0);
}

PPDL_API int ppdl_infer_batch(ppdl_ctx *c, const float *images, int n, const int32_t *ori_hw,
                              ppdl_result *res) {
    if (!c || !images || !ori_hw || !res || n < 1 || n > c->m->Bmax) return 1;
    for (int i = 0; i < n; i++)
        if (ori_hw[2 * i] <= 0 || ori_hw[2 * i + 1] <= 0) return 1;
    int rc = enqueue(c, images, false, n, ori_hw);
    if (rc) return rc;
    ppdl::Model &m = *c->m;
    cudaMemcpyAsync(c->h_dets, m.dets, sizeof(float) * ppdl::kNQ * 7 * n, cudaMemcpyDeviceToHost,
                    m.st);
    cudaMemcpyAsync(c->h_masks, m.masks, sizeof(int32_t) * (size_t)ppdl::kNQ * ppdl::kMaskPix * n,
                    cudaMemcpyDeviceToHost, m.st);
    if (cudaStreamSynchronize(m.st) != cudaSuccess) {
        fprintf(stderr, "ppdl: graph compute failed: %s\n", cudaGetErrorString(cudaGetLastError()));
        return 2;
    }
    if (ppdl::tc_error_fetch_and_clear()) {
        fprintf(stderr, "ppdl: tensor-core GEMM gave up waiting (device error flag set)\n");
        return 2;
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->e0, c->e1);
    c->computed = true;
    for (int i = 0; i < n; i++) {
        res[i].dets = c->h_dets + (size_t)i * ppdl::kNQ * 7;
        res[i].num_dets = ppdl::kNQ;
        res[i].masks = c->h_masks + (size_t)i * ppdl::kNQ * ppdl::kMaskPix;
        res[i].infer_ms = ms;
    }
    return 0;
}

PPDL_API int ppdl_infer(ppdl_ctx *c, const float *image_chw, int ori_h, int ori_w,
                        ppdl_result *result) {
    if (!c || !image_chw || !result) return 1;
    if (ori_h <= 0 || ori_w <= 0) return 1;
    const int32_t hw[2] = {ori_h, ori_w};
    return ppdl_infer_batch(c, image_chw, 1, hw, result);
}

PPDL_API int ppdl_infer_device(ppdl_ctx *c, const float *d_images, int n, const int32_t *ori_hw) {
    if (!c || !d_images || !ori_hw || n < 1 || n > c->m->Bmax) return 1;
    for (int i = 0; i < n; i++)
        if (ori_hw[2 * i] <= 0 || ori_hw[2 * i + 1] <= 0) return 1;
    const int rc = enqueue(c, d_images, true, n, ori_hw);
    if (!rc) c->computed = true;
    return rc;
}

PPDL_API int ppdl_device_outputs(ppdl_ctx *c, const float **d_dets, const int32_t **d_masks) {
    if (!c || !c->computed) return 1;
    if (d_dets) *d_dets = c->m->dets;
    if (d_masks) *d_masks = c->m->masks;
    return 0;
}

PPDL_API int ppdl_sync(ppdl_ctx *c) {
    if (!c) return 1;
    cudaSetDevice(c->m->dev);
    if (cudaStreamSynchronize(c->m->st) != cudaSuccess) return 2;
    return ppdl::tc_error_fetch_and_clear() ? 2 : 0;
}

PPDL_API int ppdl_infer_device_bits(ppdl_ctx *c, const float *d_images, int n,
                                   const int32_t *ori_hw) {
    if (!c || !d_images || !ori_hw || n < 1 || n > c->m->Bmax) return 1;
    for (int i = 0; i < n; i++)
        if (ori_hw[2 * i] <= 0 || ori_hw[2 * i + 1] <= 0) return 1;
    const int rc = enqueue(c, d_images, true, n, ori_hw, false);
    if (!rc) c->computed = true;
    return rc;
}

PPDL_API int ppdl_device_mask_bits(ppdl_ctx *c, const uint32_t **d_bits) {
    if (!c || !c->computed || !d_bits) return 1;
    *d_bits = c->m->mask_bits;
    return 0;
}

namespace {

bool pipe_setup(ppdl_ctx *c) {
    PpdlPipe &p = c->pipe;
    if (p.ready) return true;
    const int B = c->m->Bmax;
    const size_t img = (size_t)3 * ppdl::kImg * ppdl::kImg * sizeof(float) * B;
    const size_t dets = sizeof(float) * ppdl::kNQ * 7 * B;
    const size_t bits = sizeof(uint32_t) * (size_t)ppdl::kNQ * ppdl::kMaskWords * B;
    bool ok = cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking) == cudaSuccess;
    for (int s = 0; s < 2 && ok; s++) {
        ok = cudaMalloc(&p.d_in[s], img) == cudaSuccess &&
             cudaMalloc(&p.d_hw[s], sizeof(int32_t) * 2 * B) == cudaSuccess &&
             cudaMalloc(&p.d_dets[s], dets) == cudaSuccess &&
             cudaMalloc(&p.d_bits[s], bits) == cudaSuccess &&
             cudaHostAlloc(&p.h_dets[s], dets, 0) == cudaSuccess &&
             cudaHostAlloc(&p.h_bits[s], bits, 0) == cudaSuccess;
        for (cudaEvent_t *e : {&p.in_ready[s], &p.in_free[s], &p.out_ready[s], &p.out_done[s]})
            ok = ok && cudaEventCreateWithFlags(e, cudaEventDisableTiming) == cudaSuccess;
        ok = ok && cudaEventCreate(&p.t0[s]) == cudaSuccess && cudaEventCreate(&p.t1[s]) == cudaSuccess;
    }
    if (!ok) {
        cudaGetLastError();
        pipe_release(p);
        fprintf(stderr, "ppdl: pipeline buffer allocation failed\n");
        return false;
    }
    p.ready = true;
    return true;
}

}  // namespace

PPDL_API int ppdl_submit_batch(ppdl_ctx *c, const float *images, int n, const int32_t *ori_hw,
                               int64_t *ticket) {
    if (!c || !images || !ori_hw || !ticket || n < 1 || n > c->m->Bmax) return 1;
    for (int i = 0; i < n; i++)
        if (ori_hw[2 * i] <= 0 || ori_hw[2 * i + 1] <= 0) return 1;
    ppdl::Model &m = *c->m;
    cudaSetDevice(m.dev);
    if (!pipe_setup(c)) return 2;
    PpdlPipe &p = c->pipe;
    const long long t = p.next;
    const int s = (int)(t & 1);
    // the slot's previous batch (ticket t - 2) must have left its host
    // buffers: results of ticket t stay valid until ticket t + 2 is submitted
    if (p.ticket_of[s] >= 0 && cudaEventSynchronize(p.out_done[s]) != cudaSuccess) return 2;
    const size_t img_bytes = (size_t)3 * ppdl::kImg * ppdl::kImg * sizeof(float) * n;
    // copy-in stream: pages into the slot's staging buffer once the forward
    // of ticket t - 2 has taken them (in_free)
    bool ok = (p.ticket_of[s] < 0 || cudaStreamWaitEvent(p.h2d, p.in_free[s], 0) == cudaSuccess) &&
              cudaMemcpyAsync(p.d_in[s], images, img_bytes, cudaMemcpyHostToDevice, p.h2d) ==
                  cudaSuccess &&
              cudaMemcpyAsync(p.d_hw[s], ori_hw, sizeof(int32_t) * 2 * n, cudaMemcpyHostToDevice,
                              p.h2d) == cudaSuccess &&
              cudaEventRecord(p.in_ready[s], p.h2d) == cudaSuccess;
    // compute stream: staging -> the forward's input, the forward (its
    // CUDA graph), dets + packed masks -> the slot's device output copy
    ok = ok && cudaStreamWaitEvent(m.st, p.in_ready[s], 0) == cudaSuccess &&
         cudaMemcpyAsync(m.img.p, p.d_in[s], img_bytes, cudaMemcpyDeviceToDevice, m.st) ==
             cudaSuccess &&
         cudaMemcpyAsync(m.ori_hw, p.d_hw[s], sizeof(int32_t) * 2 * n, cudaMemcpyDeviceToDevice,
                         m.st) == cudaSuccess &&
         cudaEventRecord(p.in_free[s], m.st) == cudaSuccess &&
         cudaEventRecord(p.t0[s], m.st) == cudaSuccess;
    if (!ok) return 2;
    m.nb = n;
    if (m.run(n) != ppdl::OK) {
        fprintf(stderr, "ppdl: forward launch failed: %s\n", cudaGetErrorString(cudaGetLastError()));
        return 2;
    }
    const size_t dets_bytes = sizeof(float) * ppdl::kNQ * 7 * n;
    const size_t bits_bytes = sizeof(uint32_t) * (size_t)ppdl::kNQ * ppdl::kMaskWords * n;
    ok = cudaEventRecord(p.t1[s], m.st) == cudaSuccess &&
         cudaMemcpyAsync(p.d_dets[s], m.dets, dets_bytes, cudaMemcpyDeviceToDevice, m.st) ==
             cudaSuccess &&
         cudaMemcpyAsync(p.d_bits[s], m.mask_bits, bits_bytes, cudaMemcpyDeviceToDevice, m.st) ==
             cudaSuccess &&
         cudaEventRecord(p.out_ready[s], m.st) == cudaSuccess &&
         // copy-out stream: the slot's outputs to its pinned host buffers
         cudaStreamWaitEvent(p.d2h, p.out_ready[s], 0) == cudaSuccess &&
         cudaMemcpyAsync(p.h_dets[s], p.d_dets[s], dets_bytes, cudaMemcpyDeviceToHost, p.d2h) ==
             cudaSuccess &&
         cudaMemcpyAsync(p.h_bits[s], p.d_bits[s], bits_bytes, cudaMemcpyDeviceToHost, p.d2h) ==
             cudaSuccess &&
         cudaEventRecord(p.out_done[s], p.d2h) == cudaSuccess;
    if (!ok) return 2;
    p.ticket_of[s] = t;
    p.n_of[s] = n;
    p.next = t + 1;
    *ticket = t;
    c->computed = true;
    c->last_n = n;
    return 0;
}

PPDL_API int ppdl_wait_batch(ppdl_ctx *c, int64_t ticket, ppdl_result_bits *res) {
    if (!c || !res || ticket < 0 || !c->pipe.ready) return 1;
    PpdlPipe &p = c->pipe;
    const int s = (int)(ticket & 1);
    if (p.ticket_of[s] != ticket) return 1;  // never submitted, or already overwritten
    cudaSetDevice(c->m->dev);
    if (cudaEventSynchronize(p.out_done[s]) != cudaSuccess) {
        fprintf(stderr, "ppdl: pipelined batch failed: %s\n",
                cudaGetErrorString(cudaGetLastError()));
        return 2;
    }
    if (ppdl::tc_error_fetch_and_clear()) {
        fprintf(stderr, "ppdl: tensor-core GEMM gave up waiting (device error flag set)\n");
        return 2;
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, p.t0[s], p.t1[s]);
    for (int i = 0; i < p.n_of[s]; i++) {
        res[i].dets = p.h_dets[s] + (size_t)i * ppdl::kNQ * 7;
        res[i].num_dets = ppdl::kNQ;
        res[i].mask_bits = p.h_bits[s] + (size_t)i * ppdl::kNQ * ppdl::kMaskWords;
        res[i].infer_ms = ms;
    }
    return 0;
}

PPDL_API void ppdl_expand_mask_bits(const uint32_t *bits, int32_t *masks, int n_dets) {
    if (!bits || !masks || n_dets <= 0) return;
    const long long words = (long long)n_dets * ppdl::kMaskWords;
    for (long long w = 0; w < words; w++) {
        const uint32_t v = bits[w];
        int32_t *o = masks + w * 32;
        for (int i = 0; i < 32; i++) o[i] = (int32_t)((v >> i) & 1u);
    }
}

PPDL_API int ppdl_dump(ppdl_ctx *c, const char *dir) {
    if (!c || !dir) return 1;
    ppdl::Model &m = *c->m;
    if (!m.dumps || m.dump_list.empty()) {
        fprintf(stderr, "ppdl: dumps not enabled\n");
        return 1;
    }
    if (!c->computed) {
        fprintf(stderr, "ppdl: no inference to dump\n");
        return 1;
    }
    cudaSetDevice(m.dev);
    cudaStreamSynchronize(m.st);
    mkdir(dir, 0755);
    FILE *mf = fopen((std::string(dir) + "/shapes.txt").c_str(), "w");
    if (!mf) return 1;
    for (auto &d : m.dump_list) {
        std::vector<char> buf(d.bytes);
        cudaMemcpy(buf.data(), d.p, d.bytes, cudaMemcpyDeviceToHost);
        write_file(std::string(dir) + "/" + d.name + ".bin", buf.data(), buf.size());
        fprintf(mf, "%s %s %lld %lld %lld %lld\n", d.name.c_str(), d.type, (long long)d.ne[0],
                (long long)d.ne[1], (long long)d.ne[2], (long long)d.ne[3]);
    }
    fclose(mf);
    return 0;
}

PPDL_API int ppdl_dump_raw(ppdl_ctx *c, const char *pfx) {
    if (!c || !pfx) return 1;
    if (!c->computed) {
        fprintf(stderr, "ppdl: no inference to dump\n");
        return 1;
    }
    ppdl::Model &m = *c->m;
    cudaSetDevice(m.dev);
    if (cudaStreamSynchronize(m.st) != cudaSuccess) return 2;
    std::vector<float> lg(ppdl::kNQ * ppdl::kNC), bx(ppdl::kNQ * 4), od(ppdl::kNQ * ppdl::kNQ);
    std::vector<int32_t> sl(ppdl::kNQ), tk(ppdl::kNQ);
    cudaMemcpy(lg.data(), m.logits.p, lg.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(tk.data(), m.enc_topk, tk.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(bx.data(), m.boxes.p, bx.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(od.data(), m.order.p, od.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(sl.data(), m.sel, sl.size() * 4, cudaMemcpyDeviceToHost);
    const std::string p(pfx);
    bool okw = write_file(p + "logits.bin", lg.data(), lg.size() * 4) &&
               write_file(p + "boxes.bin", bx.data(), bx.size() * 4) &&
               write_file(p + "order.bin", od.data(), od.size() * 4) &&
               write_file(p + "sel.bin", sl.data(), sl.size() * 4) &&
               write_file(p + "topk.bin", tk.data(), tk.size() * 4);
    return okw ? 0 : 1;
}

PPDL_API void *ppdl_stream(ppdl_ctx *c) { return c ? (void *)c->m->st : nullptr; }

PPDL_API int ppdl_profile_timeline(ppdl_ctx *c, int n, float *end_ms, int32_t *lane, int max) {
    if (!c || !end_ms || !lane || max <= 0 || n < 1 || n > c->m->Bmax || !c->computed) return -1;
    ppdl::Model &m = *c->m;
    cudaSetDevice(m.dev);
    const int ns = (int)m.plan.size();
    std::vector<cudaEvent_t> ev(ns + 1);
    for (auto &e : ev) cudaEventCreate(&e);
    m.nb = n;
    // the forward on its lanes, captured with an "external" event-record
    // node after every step on the step's own lane, replayed twice (the
    // second timed): end time of each step from the start of the forward
    int rc = 0;
    cudaGraph_t gr = nullptr;
    cudaGraphExec_t ge = nullptr;
    bool graphed = false;
    if (cudaStreamBeginCapture(m.st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        bool ok = cudaEventRecordWithFlags(ev[0], m.st, cudaEventRecordExternal) == cudaSuccess;
        ok = ok && m.exec([&](int i) {
            return cudaEventRecordWithFlags(ev[i + 1], m.st, cudaEventRecordExternal) ==
                   cudaSuccess;
        }) == ppdl::OK;
        if (cudaStreamEndCapture(m.st, &gr) == cudaSuccess && ok &&
            cudaGraphInstantiate(&ge, gr, 0) == cudaSuccess)
            graphed = cudaGraphLaunch(ge, m.st) == cudaSuccess &&
                      cudaGraphLaunch(ge, m.st) == cudaSuccess;
    }
    cudaGetLastError();
    if (!graphed || cudaStreamSynchronize(m.st) != cudaSuccess) rc = -1;
    int w = 0;
    if (rc == 0)
        for (int i = 0; i < ns && w < max; i++, w++) {
            cudaEventElapsedTime(&end_ms[w], ev[0], ev[i + 1]);
            lane[w] = m.plan[i].lane;
        }
    if (ge) cudaGraphExecDestroy(ge);
    if (gr) cudaGraphDestroy(gr);
    for (auto &e : ev) cudaEventDestroy(e);
    return rc == 0 ? w : -1;
}

PPDL_API int ppdl_profile_steps(ppdl_ctx *c, int n, ppdl_step_stat *out, int max) {
    if (!c || !out || max <= 0 || n < 1 || n > c->m->Bmax || !c->computed) return -1;
    ppdl::Model &m = *c->m;
    cudaSetDevice(m.dev);
    const int ns = (int)m.plan.size();
    std::vector<cudaEvent_t> ev(ns + 1);
    for (auto &e : ev) cudaEventCreate(&e);
    m.nb = n;
    // the steps with an event after each, captured into a CUDA graph and
    // replayed (twice, the second timed), so that the times are device time
    // without the host's launch gaps; eager if the capture fails
    // (inside a capture only an "external" record becomes an event-record
    // node; a plain one would merely mark a dependency)
    auto enqueue = [&](unsigned flags) -> bool {
        if (cudaEventRecordWithFlags(ev[0], m.st, flags) != cudaSuccess) return false;
        for (int i = 0; i < ns; i++)
            if (m.plan[i].fn() != ppdl::OK ||
                cudaEventRecordWithFlags(ev[i + 1], m.st, flags) != cudaSuccess)
                return false;
        return true;
    };
    int rc = 0;
    cudaGraph_t gr = nullptr;
    cudaGraphExec_t ge = nullptr;
    bool graphed = false;
    if (cudaStreamBeginCapture(m.st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        const bool ok = enqueue(cudaEventRecordExternal);
        if (cudaStreamEndCapture(m.st, &gr) == cudaSuccess && ok &&
            cudaGraphInstantiate(&ge, gr, 0) == cudaSuccess)
            graphed = cudaGraphLaunch(ge, m.st) == cudaSuccess &&
                      cudaGraphLaunch(ge, m.st) == cudaSuccess;
    }
    cudaGetLastError();
    if (!graphed && !enqueue(cudaEventRecordDefault)) rc = -1;
    if (cudaStreamSynchronize(m.st) != cudaSuccess) rc = -1;
    int w = 0;
    if (rc == 0) {
        for (int i = 0; i < ns && w < max; i++, w++) {
            ppdl_step_stat &s = out[w];
            memset(s.name, 0, sizeof s.name);
            strncpy(s.name, m.plan[i].name.c_str(), sizeof s.name - 1);
            s.kind = m.plan[i].kind;
            cudaEventElapsedTime(&s.ms, ev[i], ev[i + 1]);
            s.flops = m.plan[i].flops;
            s.bytes = m.plan[i].bytes;
        }
    }
    if (ge) cudaGraphExecDestroy(ge);
    if (gr) cudaGraphDestroy(gr);
    for (auto &e : ev) cudaEventDestroy(e);
    return rc == 0 ? w : -1;
}

PPDL_API void ppdl_free(ppdl_ctx *c) { ctx_release(c); }

}  // extern "C"
