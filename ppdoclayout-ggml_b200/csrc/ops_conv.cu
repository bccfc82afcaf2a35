// ops_conv.cu — conv-family op ids of the operator ABI (3, 4, 10, 11, 12).
//
// Same tensors and op_params encodings as the reference's ggml hook
// (patches/ggml-ppdl.patch:632-718, 778-812):
//   op 3  K==1 conv as one GEMM writing CHW, weights ".wr" (1, IC, OC)
//   op 4  direct conv (K,S,PAD,ACT) with fused bias/act, weights ".wr"
//         (K*K, IC, OC) — here an implicit GEMM over the tap-major k order
//   op 10 Winograd F(4,3) input transform of an already padded tensor
//   op 12 36-plane madd with ".wg4" (36, IC, OC)
//   op 11 output transform + bias + act
// The ggml ne[3] (ne[2] for the plane tensors' page count) carries pages.
//
// Ops 3 and 12 run on the 3xTF32 tensor-core GEMM.  A hook sees only its
// node's tensors and cannot allocate, so the TF32 halves of the weight go to
// the library's static split array (the one ppdl_gemm_tf32x3_static uses,
// 2^21 weights per half) in chunks of output channels (op 3) or Winograd
// planes (op 12), each chunk split and multiplied in stream order; calls
// whose GPU work overlaps on one device race on that array.  A GEMM whose
// operands TMA cannot describe (IC not a multiple of 4) keeps the SIMT
// FFMA GEMM.
#include <cstdio>

#include "conv.h"
#include "gemm.h"
#include "gemm_tc.h"
#include "ops_internal.h"

namespace ppdl {

float *static_split_workspace(long long *cap);

namespace {

long long nel(const ppdl_tensor &t) { return t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]; }

int code(Status s) {
    switch (s) {
        case OK: return PPDL_OK;
        case ERR_UNSUPPORTED: return PPDL_ERR_UNSUPPORTED;
        case ERR_SHAPE: return PPDL_ERR_SHAPE;
        default: return PPDL_ERR_CUDA;
    }
}

// C[z](m, n) for n in [0, N) as chunks of output columns whose split
// weights fit the static array; w points at the weight with element
// (plane p, k, n) at w[p * pstride + k * ldw + n] (the ggml ".wr"/".wg4"
// layouts), A: M-major, one z per (page, plane).  Returns false (nothing
// launched) when the shapes cannot use the tensor cores.
bool tc_chunked(const float *A, int M, int K, long long lda, long long a_bs, int planes, int pages,
                const float *w, long long ldw, long long pstride, int N, float *C,
                long long ldc_n, long long c_bs, cudaStream_t st, Status *out) {
    long long cap = 0;
    float *ws = static_split_workspace(&cap);
    if (!ws || K % 4) return false;
    float *hi = ws, *lo = ws + cap;
    // chunk: all output columns of as many planes as fit, else the columns
    // of one plane in multiples of 16
    const long long per_plane = (long long)N * K;
    int pc = (int)(cap / per_plane);
    int nc = N;
    if (pc < 1) {
        pc = 1;
        nc = (int)(cap / K) / 16 * 16;
        if (nc < 16) return false;
    }
    if (pc > planes) pc = planes;
    // plan every chunk before launching anything
    struct Chunk { int p0, np, n0, nn, b; };
    const int n_pchunks = (planes + pc - 1) / pc, n_nchunks = (N + nc - 1) / nc;
    for (int pi = 0; pi < n_pchunks; pi++)
        for (int ni = 0; ni < n_nchunks; ni++) {
            const int p0 = pi * pc, np = planes - p0 < pc ? planes - p0 : pc;
            const int n0 = ni * nc, nn = N - n0 < nc ? N - n0 : nc;
            // one split of the chunk's weights, then one GEMM per page (the
            // planes of a page are consecutive z)
            if (launch_kmajor_split(w + (long long)p0 * pstride + n0, hi, lo, np, K, (int)ldw,
                                    pstride, nn, st) != OK) {
                *out = ERR_CUDA;
                return true;
            }
            for (int b = 0; b < pages; b++) {
                const long long z0 = (long long)b * planes + p0;
                TcEpilogue e;
                e.C = C + z0 * c_bs + (long long)n0 * ldc_n;
                e.ldc_m = 1; e.ldc_n = ldc_n; e.c_bs = c_bs;
                TcGemm g;
                const float *Az = A + z0 * a_bs;
                if (!tc_gemm_plan(&g, M, nn, K, np, Az, 1, lda, a_bs, hi, lo, np, e) &&
                    !tc_gemm_plan_rows(&g, M, nn, K, np, Az, lda, a_bs, hi, lo, e, np)) {
                    // only the first chunk can fail (same strides for all):
                    // nothing has been multiplied yet
                    if (pi == 0 && ni == 0 && b == 0) return false;
                    *out = ERR_SHAPE;
                    return true;
                }
                const Status s = launch_tc_gemm(g, st);
                if (s != OK) {
                    *out = s;
                    return true;
                }
            }
        }
    *out = OK;
    return true;
}

}  // namespace

bool ops_ext_provided(int id) {
    return id == PPDL_OP_CONV || id == PPDL_OP_CONVDIRECT || id == PPDL_OP_WG4_INPUT ||
           id == PPDL_OP_WG4_OUTPUT || id == PPDL_OP_WG4_MADD;
}

bool ops_ext_launch(const ppdl_op_desc *d, cudaStream_t st, int *status, char *err,
                    size_t err_len) {
    const int32_t *p = d->op_params;
    const ppdl_tensor &dst = d->dst, &s0 = d->src[0], &s1 = d->src[1], &s2 = d->src[2];
    auto bad = [&](const char *msg) {
        snprintf(err, err_len, "%s", msg);
        *status = PPDL_ERR_SHAPE;
        return true;
    };
    switch (p[13]) {
        case PPDL_OP_CONV: {
            const int K = p[14] & 0xFF;
            if (p[15] != 0 || K != 1) {
                snprintf(err, err_len, "op 3: only the K==1 CHW form is provided");
                *status = PPDL_ERR_UNSUPPORTED;
                return true;
            }
            const long long IW = s0.ne[0], IH = s0.ne[1], IC = s0.ne[2], B = s0.ne[3];
            const long long OC = dst.ne[2];
            if (dst.ne[0] != IW || dst.ne[1] != IH || dst.ne[3] != B || s1.ne[0] != OC ||
                s1.ne[1] != IC || nel(s1) != OC * IC)
                return bad("op 3: x / .wr / dst shapes disagree");
            {
                // tensor cores: A = x (pixels x channels, M-major), B(oc, ic) = wr[ic][oc]
                Status ts = OK;
                if (tc_chunked((const float *)s0.data, (int)(IW * IH), (int)IC, IW * IH,
                               IW * IH * IC, 1, (int)B, (const float *)s1.data, OC, 0, (int)OC,
                               (float *)dst.data, IW * IH, IW * IH * OC, st, &ts)) {
                    *status = code(ts);
                    return true;
                }
            }
            GemmArgs g;  // dst[oc][p] = sum_ic wr[ic][oc] x[ic][p]
            g.M = (int)OC; g.N = (int)(IW * IH); g.K = (int)IC; g.batch = (int)B;
            g.A = {(const float *)s1.data, 1, OC};
            g.B = {(const float *)s0.data, IW * IH, 1, 1, IW * IH * IC, 0};
            g.C = (float *)dst.data; g.ldc_m = IW * IH; g.ldc_n = 1; g.c_bs_hi = IW * IH * OC;
            *status = code(launch_gemm_simt(g, st));
            return true;
        }
        case PPDL_OP_CONVDIRECT: {
            const int K = p[14] & 0xFF, S = (p[14] >> 8) & 0xFF, P = (p[14] >> 16) & 0xFF;
            const int act = (p[14] >> 24) & 0xFF;
            const bool form_ok = (K == 3 && S == 1 && P == 1) || (K == 3 && S == 2 && P == 1) ||
                                 (K == 2 && S == 1 && P == 0) || (K == 1 && S == 1 && P == 0);
            if (!form_ok || act > 2) return bad("op 4: unsupported K/S/PAD/ACT combination");
            const long long IW = s0.ne[0], IH = s0.ne[1], IC = s0.ne[2], B = s0.ne[3];
            const long long OW = dst.ne[0], OH = dst.ne[1], OC = dst.ne[2];
            if (OW != (IW + 2 * P - K) / S + 1 || OH != (IH + 2 * P - K) / S + 1 ||
                dst.ne[3] != B || s1.ne[0] != OC || s1.ne[1] != IC || s1.ne[2] != K * K ||
                nel(s2) != OC)
                return bad("op 4: x / .wr / bias / dst shapes disagree");
            GemmArgs g;  // k = (kh*K + kw)*IC + ic, A(oc, k) = wr[k][oc]
            g.M = (int)OC; g.N = (int)(OW * OH); g.K = (int)(IC * K * K); g.batch = (int)B;
            g.A = {(const float *)s1.data, 1, OC};
            g.B = {(const float *)s0.data, 0, 0, 1, IW * IH * IC, 0};
            g.conv = {K, S, P, (int)IH, (int)IW, (int)OW, (int)IC, 1};
            g.C = (float *)dst.data; g.ldc_m = OW * OH; g.ldc_n = 1; g.c_bs_hi = OW * OH * OC;
            g.bias = (const float *)s2.data; g.bias_mode = 1; g.act = act;
            *status = code(launch_gemm_simt(g, st));
            return true;
        }
        case PPDL_OP_WG4_INPUT: {
            const long long IWp = s0.ne[0], IHp = s0.ne[1], IC = s0.ne[2], B = s0.ne[3];
            const int T = p[14], TH = p[15];
            if (T <= 0 || TH <= 0 || T % TH) return bad("op 10: op_params T/TH invalid");
            const int TW = T / TH;
            if (IWp < 4LL * TW + 2 || IHp < 4LL * TH + 2)
                return bad("op 10: padded input smaller than the tile grid");
            if (dst.ne[0] != T || dst.ne[1] != IC || dst.ne[2] != 36 || dst.ne[3] != B)
                return bad("op 10: dst must be ne(T, IC, 36, B)");
            *status = code(launch_wg4_input((const float *)s0.data, IWp * IHp * IC,
                                            (float *)dst.data, (int)IC, (int)IHp, (int)IWp, TW, TH,
                                            0, (int)B, st));
            return true;
        }
        case PPDL_OP_WG4_MADD: {
            const long long T = dst.ne[0], OC = dst.ne[1], IC = s0.ne[1], B = dst.ne[3];
            if (s0.ne[0] != T || s0.ne[2] != 36 || s0.ne[3] != B || dst.ne[2] != 36 ||
                s1.ne[0] != OC || s1.ne[1] != IC || s1.ne[2] != 36)
                return bad("op 12: dt / .wg4 / yt shapes disagree");
            {
                // tensor cores, per plane p: A(t, ic) = dt[b][p][ic][t],
                // B(oc, ic) = wg4[p][ic][oc], yt[b][p][oc][t]
                Status ts = OK;
                if (tc_chunked((const float *)s0.data, (int)T, (int)IC, T, IC * T, 36, (int)B,
                               (const float *)s1.data, OC, IC * OC, (int)OC, (float *)dst.data, T,
                               OC * T, st, &ts)) {
                    *status = code(ts);
                    return true;
                }
            }
            GemmArgs g;
            g.M = (int)OC; g.N = (int)T; g.K = (int)IC; g.batch = (int)(B * 36);
            g.A = {(const float *)s1.data, 1, OC, 36, 0, IC * OC};
            g.B = {(const float *)s0.data, T, 1, 1, IC * T, 0};
            g.C = (float *)dst.data; g.ldc_m = T; g.ldc_n = 1; g.c_bs_hi = OC * T;
            *status = code(launch_gemm_simt(g, st));
            return true;
        }
        case PPDL_OP_WG4_OUTPUT: {
            const long long OW = dst.ne[0], OH = dst.ne[1], OC = dst.ne[2], B = dst.ne[3];
            const int TW = p[15];
            const long long T = ((OW + 3) / 4) * ((OH + 3) / 4);
            if (TW <= 0 || T % TW) return bad("op 11: op_params TW invalid");
            const int TH = (int)(T / TW);
            if (s0.ne[0] != T || s0.ne[1] != OC || s0.ne[2] != 36 || s0.ne[3] != B ||
                nel(s1) != OC || p[14] < 0 || p[14] > 2)
                return bad("op 11: yt / bias / dst shapes or act disagree");
            *status = code(launch_wg4_output((const float *)s0.data, (const float *)s1.data,
                                             (float *)dst.data, OW * OH * OC, nullptr, 0, 0,
                                             (int)OC, (int)OH, (int)OW, TW, TH, p[14], (int)B, st));
            return true;
        }
        default:
            return false;
    }
}

}  // namespace ppdl
