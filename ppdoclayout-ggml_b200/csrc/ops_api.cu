// ops_api.cu — the operator-level C ABI (include/ppdl_ops.h).
//
// Replaces the reference's ggml hook pair ggml_cuda_compute_forward_ppdl /
// ggml_cuda_supports_ppdl_op (patches/ggml-ppdl.patch:612-817, 908-917): the
// same op ids, the same op_params[14]/[15] encodings, the same tensor
// layouts.  Where the reference aborts on a shape violation (GGML_ASSERT)
// this layer returns PPDL_ERR_SHAPE with a message instead; where the
// reference hook returns false (unknown id) this returns
// PPDL_ERR_UNSUPPORTED.
#include <cstdio>
#include <cstring>

#include "../../include/ppdl_ops.h"
#include "kernels.h"
#include "conv.h"
#include "dec.h"
#include "gemm_tc.h"
#include "ops_internal.h"

namespace {

thread_local char g_err[256] = "";

int fail(int code, const char *fmt, long long a = 0, long long b = 0) {
    snprintf(g_err, sizeof g_err, fmt, a, b);
    return code;
}

long long nel(const ppdl_tensor &t) { return t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]; }

int to_status(ppdl::Status s) {
    switch (s) {
        case ppdl::OK: return PPDL_OK;
        case ppdl::ERR_UNSUPPORTED: return fail(PPDL_ERR_UNSUPPORTED, "unsupported op form");
        case ppdl::ERR_SHAPE: return fail(PPDL_ERR_SHAPE, "shape, size or alignment violation");
        default: {
            snprintf(g_err, sizeof g_err, "CUDA launch failed");
            return PPDL_ERR_CUDA;
        }
    }
}

bool provided(int id) {
    switch (id) {
        case PPDL_OP_MASKBOX: case PPDL_OP_MSDEF: case PPDL_OP_BIASACT: case PPDL_OP_COPY:
        case PPDL_OP_TOPK:
            return true;
        default:
            return ppdl::ops_ext_provided(id);
    }
}

}  // namespace

namespace ppdl {
// Lets other entry points of this library report through ppdl_op_last_error.
void set_op_error(const char *msg) { snprintf(g_err, sizeof g_err, "%s", msg); }
}  // namespace ppdl

extern "C" {

PPDL_OPS_API int ppdl_op_supported(const ppdl_op_desc *d) {
    if (!d || (uint32_t)d->op_params[12] != PPDL_MAGIC) return 0;
    const int id = d->op_params[13];
    if (id == PPDL_OP_CONV && d->op_params[15] != 0) return 0;
    return provided(id) ? 1 : 0;
}

PPDL_OPS_API const char *ppdl_op_last_error(void) { return g_err; }

PPDL_OPS_API int ppdl_op_device_error(void) { return ppdl::tc_error_fetch_and_clear() ? 1 : 0; }

PPDL_OPS_API int ppdl_gemm_tf32x3_presplit(int M, int N, int K, int batch, const float *A,
                                           int a_m_major, long long lda, long long a_bs,
                                           const float *b_split, float *C, long long ldc_m,
                                           long long ldc_n, long long c_bs, void *stream);

PPDL_OPS_API int ppdl_gemm_tf32x3(int M, int N, int K, int batch, const float *A, int a_m_major,
                                  long long lda, long long a_bs, const float *B, float *b_split,
                                  float *C, long long ldc_m, long long ldc_n, long long c_bs,
                                  void *stream) {
    g_err[0] = 0;
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || !A || !B || !b_split || !C)
        return fail(PPDL_ERR_SHAPE, "gemm: bad sizes or null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    ppdl::Status s = ppdl::launch_tf32_split(B, b_split, b_split + (long long)N * K,
                                             (long long)N * K, st);
    if (s != ppdl::OK) return to_status(s);
    return ppdl_gemm_tf32x3_presplit(M, N, K, batch, A, a_m_major, lda, a_bs, b_split, C, ldc_m,
                                     ldc_n, c_bs, stream);
}

PPDL_OPS_API int ppdl_depthwise_conv2d(const float *x, int batch, int C, int H, int W,
                                       long long x_bs, const float *weight, const float *bias,
                                       int K, int S, int P, int act, float *y, long long y_bs,
                                       void *stream) {
    g_err[0] = 0;
    if (!x || !weight || !y || batch <= 0 || C <= 0 || H <= 0 || W <= 0 || act < 0 || act > 3)
        return fail(PPDL_ERR_SHAPE, "depthwise conv: bad sizes, activation or null pointer");
    if (!((K == 3 || K == 5) && (S == 1 || S == 2)))
        return fail(PPDL_ERR_UNSUPPORTED, "depthwise conv: K %lld, stride %lld (3 or 5, 1 or 2)", K,
                    S);
    return to_status(ppdl::launch_dwconv(x, x_bs, weight, bias, y, y_bs, C, H, W, K, S, P, act,
                                         batch, (cudaStream_t)stream));
}

PPDL_OPS_API int ppdl_conv2d_direct(const float *x, int batch, int IC, int H, int W,
                                    long long x_bs, const float *weight, const float *bias,
                                    int OC, int K, int S, int P, int OH, int OW, int act,
                                    float *y, long long y_bs, void *stream) {
    g_err[0] = 0;
    if (!x || !weight || !y || batch <= 0 || H <= 0 || W <= 0 || OH <= 0 || OW <= 0 || act < 0 ||
        act > 3 || P < 0 || P >= K)
        return fail(PPDL_ERR_SHAPE, "conv2d_direct: bad sizes, activation or null pointer");
    if (!ppdl::conv_direct_ok(IC, OC, K, S))
        return fail(PPDL_ERR_UNSUPPORTED,
                    "conv2d_direct: needs OC <= 32, IC*K*K <= 128, K 2..3, S 1..2");
    if ((long long)(OH - 1) * S - P >= H || (long long)(OW - 1) * S - P >= W)
        return fail(PPDL_ERR_SHAPE, "conv2d_direct: output %dx%d larger than the input allows",
                    OH, OW);
    return to_status(ppdl::launch_conv_direct(x, x_bs, weight, bias, y, y_bs, IC, H, W, OC, K, S,
                                              P, OH, OW, act, batch, (cudaStream_t)stream));
}

PPDL_OPS_API int ppdl_attention_f32(const float *q, const float *k, const float *v, float *o,
                                    int batch, int T, int heads, int ldqk, long long bsqk,
                                    int ldvo, long long bsvo, float scale, void *stream) {
    g_err[0] = 0;
    if (!q || !k || !v || !o || batch <= 0 || T <= 0 || heads <= 0)
        return fail(PPDL_ERR_SHAPE, "attention: bad sizes or null pointer");
    const ppdl::Status s = ppdl::launch_attention(q, k, v, o, T, heads, ldqk, bsqk, ldvo, bsvo,
                                                  scale, batch, (cudaStream_t)stream);
    if (s == ppdl::ERR_SHAPE)
        return fail(PPDL_ERR_SHAPE, "attention: rows of 32-float heads need 16-byte alignment "
                                    "and strides that are multiples of 4 floats");
    return to_status(s);
}

PPDL_OPS_API long long ppdl_conv2d_tf32x3_workspace(int IC, int OC, int K) {
    if (IC <= 0 || OC <= 0 || K <= 0) return 0;
    const long long kp = (IC * K * K + 3) / 4 * 4, kb = ppdl::tc_conv_box_kdim(IC, K);
    return 2LL * OC * (kp > kb ? kp : kb);
}

PPDL_OPS_API int ppdl_conv2d_tf32x3(const float *x, int batch, int IC, int H, int W,
                                    long long x_bs, const float *weight, const float *bias,
                                    int OC, int K, int S, int P, int OH, int OW, int act,
                                    float *b_split, float *y, long long y_bs, void *stream) {
    g_err[0] = 0;
    if (!x || !weight || !b_split || !y || batch <= 0 || IC <= 0 || OC <= 0 || H <= 0 ||
        W <= 0 || OH <= 0 || OW <= 0 || act < 0 || act > 3)
        return fail(PPDL_ERR_SHAPE, "conv2d: bad sizes, activation or null pointer");
    // the last window of each axis must start inside the input (rows past
    // the bottom/right edge are the implicit zero padding)
    if ((long long)(OH - 1) * S - P >= H || (long long)(OW - 1) * S - P >= W ||
        (long long)OH * OW >= (1LL << 31))
        return fail(PPDL_ERR_SHAPE, "conv2d: output %dx%d larger than the input allows", OH, OW);
    cudaStream_t st = (cudaStream_t)stream;
    ppdl::TcEpilogue e;
    e.C = y; e.ldc_m = 1; e.ldc_n = (long long)OH * OW; e.c_bs = y_bs;
    e.bias = bias; e.act = act;
    ppdl::TcGemm g;
    // the forward's path: TMA windows of the input when its rows are 16-byte
    // multiples (K > 1), else the converter warps' gather
    if (K > 1) {
        ppdl::TcConvBox cb;
        cb.x = x; cb.x_bs = x_bs;
        cb.IC = IC; cb.H = H; cb.W = W; cb.KS = K; cb.S = S; cb.P = P; cb.OH = OH; cb.OW = OW;
        const int Kb = ppdl::tc_conv_box_kdim(IC, K);
        float *hi = b_split, *lo = b_split + (long long)OC * Kb;
        if (ppdl::tc_gemm_plan_box(&g, OC, batch, cb, hi, lo, e)) {
            const ppdl::Status s = ppdl::launch_tf32_split_box(weight, hi, lo, OC, IC, K, st);
            if (s != ppdl::OK) return to_status(s);
            return to_status(ppdl::launch_tc_gemm(g, st));
        }
    }
    const int Kc = IC * K * K, Kp = (Kc + 3) / 4 * 4;
    float *hi = b_split, *lo = b_split + (long long)OC * Kp;
    ppdl::TcGather gg;
    gg.x = x; gg.x_bs = x_bs; gg.plane = (long long)H * W;
    gg.KS = K; gg.S = S; gg.P = P; gg.H = H; gg.W = W; gg.OW = OW;
    if (!ppdl::tc_gemm_plan_gather(&g, OH * OW, OC, Kc, batch, gg, hi, lo, e))
        return fail(PPDL_ERR_SHAPE, "conv2d: geometry outside the gather (K 1..8, P < K, "
                                    "1x1 only with S=1 P=0) or misaligned b_split");
    const ppdl::Status s = ppdl::launch_tf32_split_pad(weight, hi, lo, OC, Kc, Kp, st);
    if (s != ppdl::OK) return to_status(s);
    return to_status(ppdl::launch_tc_gemm(g, st));
}

namespace {
// Winograd F(4,3) conv workspace, in floats, each part a multiple of 4:
// wg4 [36][IC][OC], hi / lo [36][OC][IC], dt [B*36][IC][Tp], yt [B*36][OC][Tp]
struct Wg4Parts {
    long long wg4, split, dt, yt;
};
Wg4Parts wg4_parts(int batch, int IC, int OC, int H, int W) {
    const long long T = (long long)((W + 3) / 4) * ((H + 3) / 4), Tp = (T + 3) / 4 * 4;
    return {36LL * IC * OC, 36LL * IC * OC, 36LL * batch * IC * Tp, 36LL * batch * OC * Tp};
}
}  // namespace

PPDL_OPS_API long long ppdl_conv3x3_wg4_workspace(int batch, int IC, int OC, int H, int W) {
    if (batch <= 0 || IC <= 0 || OC <= 0 || H <= 0 || W <= 0) return 0;
    const Wg4Parts q = wg4_parts(batch, IC, OC, H, W);
    return q.wg4 + 2 * q.split + q.dt + q.yt;
}

PPDL_OPS_API int ppdl_conv3x3_wg4_prepare(const float *weight, int IC, int OC, float *work,
                                          void *stream) {
    g_err[0] = 0;
    if (!weight || !work || IC <= 0 || OC <= 0 || IC % 4 || ((uintptr_t)work & 15))
        return fail(PPDL_ERR_SHAPE, "conv3x3 prepare: bad sizes, IC not a multiple of 4 or "
                                    "misaligned workspace");
    cudaStream_t st = (cudaStream_t)stream;
    const Wg4Parts q = wg4_parts(1, IC, OC, 1, 1);
    float *wg4 = work, *hi = wg4 + q.wg4, *lo = hi + q.split;
    ppdl::Status s = ppdl::launch_wg4_filter(weight, wg4, IC, OC, st);
    if (s == ppdl::OK) s = ppdl::launch_wg4_kmajor_split(wg4, hi, lo, IC, OC, st);
    return to_status(s);
}

PPDL_OPS_API int ppdl_conv3x3_wg4_run(const float *x, int batch, int IC, int H, int W,
                                      long long x_bs, const float *bias, int OC, int act,
                                      float *work, float *y, long long y_bs, void *stream) {
    g_err[0] = 0;
    if (!x || !work || !y || batch <= 0 || IC <= 0 || OC <= 0 || H <= 0 || W <= 0 || act < 0 ||
        act > 3)
        return fail(PPDL_ERR_SHAPE, "conv3x3: bad sizes, activation or null pointer");
    if (IC % 4 || ((uintptr_t)work & 15))
        return fail(PPDL_ERR_SHAPE, "conv3x3: IC must be a multiple of 4 and the workspace "
                                    "16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    const int TW = (W + 3) / 4, TH = (H + 3) / 4, T = TW * TH, Tp = (T + 3) / 4 * 4;
    const Wg4Parts q = wg4_parts(batch, IC, OC, H, W);
    float *wg4 = work, *hi = wg4 + q.wg4, *lo = hi + q.split, *dt = lo + q.split, *yt = dt + q.dt;
    ppdl::TcEpilogue e;
    e.C = yt; e.ldc_m = 1; e.ldc_n = Tp; e.c_bs = (long long)OC * Tp;
    ppdl::TcGemm g;
    if (!ppdl::tc_gemm_plan(&g, T, OC, IC, batch * 36, dt, 1, Tp, (long long)IC * Tp, hi, lo, 36,
                            e))
        return fail(PPDL_ERR_SHAPE, "conv3x3: the plane GEMM cannot be planned");
    ppdl::Status s = ppdl::launch_wg4_input(x, x_bs, dt, IC, H, W, TW, TH, 1, batch, st, Tp);
    if (s == ppdl::OK) s = ppdl::launch_tc_gemm(g, st);
    if (s == ppdl::OK)
        s = ppdl::launch_wg4_output(yt, bias, y, y_bs, nullptr, 0, 0, OC, H, W, TW, TH, act,
                                    batch, st, Tp);
    return to_status(s);
}

PPDL_OPS_API int ppdl_conv3x3_wg4_tf32x3(const float *x, int batch, int IC, int H, int W,
                                         long long x_bs, const float *weight, const float *bias,
                                         int OC, int act, float *work, float *y, long long y_bs,
                                         void *stream) {
    if (!x || !weight || !work || !y || batch <= 0 || IC <= 0 || OC <= 0 || H <= 0 || W <= 0 ||
        act < 0 || act > 3) {
        g_err[0] = 0;
        return fail(PPDL_ERR_SHAPE, "conv3x3: bad sizes, activation or null pointer");
    }
    const int rc = ppdl_conv3x3_wg4_prepare(weight, IC, OC, work, stream);
    if (rc != PPDL_OK) return rc;
    return ppdl_conv3x3_wg4_run(x, batch, IC, H, W, x_bs, bias, OC, act, work, y, y_bs, stream);
}

PPDL_OPS_API int ppdl_tf32_split(const float *w, long long n, float *b_split, void *stream) {
    g_err[0] = 0;
    if (!w || !b_split || n <= 0) return fail(PPDL_ERR_SHAPE, "tf32_split: bad size or pointer");
    return to_status(ppdl::launch_tf32_split(w, b_split, b_split + n, n, (cudaStream_t)stream));
}

PPDL_OPS_API int ppdl_gemm_tf32x3_presplit(int M, int N, int K, int batch, const float *A,
                                           int a_m_major, long long lda, long long a_bs,
                                           const float *b_split, float *C, long long ldc_m,
                                           long long ldc_n, long long c_bs, void *stream) {
    g_err[0] = 0;
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || !A || !b_split || !C)
        return fail(PPDL_ERR_SHAPE, "gemm: bad sizes or null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const float *hi = b_split, *lo = b_split + (long long)N * K;
    ppdl::TcEpilogue e;
    e.C = C; e.ldc_m = ldc_m; e.ldc_n = ldc_n; e.c_bs = c_bs;
    ppdl::TcGemm g;
    if (!ppdl::tc_gemm_plan(&g, M, N, K, batch, A, a_m_major ? 1 : 0, lda, a_bs, hi, lo, 1, e) &&
        !(a_m_major && ppdl::tc_gemm_plan_rows(&g, M, N, K, batch, A, lda, a_bs, hi, lo, e)))
        return fail(PPDL_ERR_SHAPE, "gemm: operands violate the TMA rules (16-byte aligned "
                                    "b_split and a_bs, K a multiple of 4; K-major A also lda)");
    return to_status(ppdl::launch_tc_gemm(g, st));
}

PPDL_OPS_API int ppdl_gemm_tf32x3_split_k(int M, int N, int K, const float *A, long long lda,
                                          const float *b_split, const float *bias,
                                          const float *res, int act, int splits, float *ws,
                                          float *C, void *stream) {
    g_err[0] = 0;
    if (M <= 0 || N <= 0 || K <= 0 || !A || !b_split || !ws || !C || act < 0 || act > 3)
        return fail(PPDL_ERR_SHAPE, "gemm split-K: bad sizes, activation or null pointer");
    ppdl::TcEpilogue e;
    e.C = C; e.ldc_m = N; e.ldc_n = 1;
    e.bias = bias; e.act = act;
    if (res) {
        e.res = res; e.res_ldm = N; e.res_ldn = 1; e.res_mode = 2;
    }
    ppdl::TcGemm g;
    if (!ppdl::tc_gemm_plan_split_k(&g, M, N, K, A, 0, lda, b_split, b_split + (long long)N * K, e,
                                    splits, ws))
        return fail(PPDL_ERR_SHAPE, "gemm split-K: K and N multiples of 4, lda too, 16-byte "
                                    "aligned operands, at least two splits of 32-wide k-blocks");
    return to_status(ppdl::launch_tc_gemm(g, (cudaStream_t)stream));
}

PPDL_OPS_API int ppdl_op_launch(const ppdl_op_desc *d, void *stream_ptr) {
    g_err[0] = 0;
    if (!d) return fail(PPDL_ERR_SHAPE, "null descriptor");
    if ((uint32_t)d->op_params[12] != PPDL_MAGIC)
        return fail(PPDL_ERR_UNSUPPORTED, "op_params[12] is not the PPDL magic");
    cudaStream_t st = (cudaStream_t)stream_ptr;
    const int32_t *p = d->op_params;
    const ppdl_tensor &dst = d->dst;
    const ppdl_tensor &s0 = d->src[0];
    switch (p[13]) {
        case PPDL_OP_MASKBOX: {
            // patch:618-622: dst ne(4, nq), src0 ne(40000, nq)
            if (dst.ne[0] != 4 || s0.ne[0] != ppdl::kMaskPix)
                return fail(PPDL_ERR_SHAPE, "mask_box: dst ne0 %lld (want 4), src ne0 %lld (want 40000)",
                            dst.ne[0], s0.ne[0]);
            const long long rows = dst.ne[1] * dst.ne[2] * dst.ne[3];
            if (s0.ne[1] * s0.ne[2] * s0.ne[3] != rows)
                return fail(PPDL_ERR_SHAPE, "mask_box: %lld src rows vs %lld dst rows",
                            s0.ne[1] * s0.ne[2] * s0.ne[3], rows);
            return to_status(ppdl::launch_mask_box((const float *)s0.data, (float *)dst.data,
                                                   (int)rows, st));
        }
        case PPDL_OP_MSDEF: {
            // patch:623-631: dst ne(256, nq), value ne(256, 13125); pages in ne[2]
            const bool canon = p[14] == 1;
            const long long nq = dst.ne[1], B = dst.ne[2] * dst.ne[3];
            if (dst.ne[0] != ppdl::kDM || s0.ne[0] != ppdl::kDM || s0.ne[1] != ppdl::kNTok)
                return fail(PPDL_ERR_SHAPE, "msdeform: dst ne0 %lld / value ne(%lld, .) mismatch",
                            dst.ne[0], s0.ne[0]);
            if (s0.ne[2] * s0.ne[3] != B || nel(d->src[1]) != 192 * nq * B ||
                nel(d->src[2]) != 96 * nq * B || (!canon && nel(d->src[3]) != 4 * nq * B))
                return fail(PPDL_ERR_SHAPE, "msdeform: operand sizes disagree with nq=%lld B=%lld",
                            nq, B);
            return to_status(ppdl::launch_msda((const float *)s0.data, (const float *)d->src[1].data,
                                               (const float *)d->src[2].data,
                                               canon ? nullptr : (const float *)d->src[3].data,
                                               (float *)dst.data, (int)nq, (int)B, canon, 192,
                                               96, st));
        }
        case PPDL_OP_BIASACT: {
            // patch:719-728: dst = act(src0 + bias[plane]), plane = ne0*ne1
            const long long n = nel(dst);
            if (nel(s0) != n) return fail(PPDL_ERR_SHAPE, "bias_act: %lld vs %lld elements", nel(s0), n);
            if (nel(d->src[1]) != dst.ne[2])
                return fail(PPDL_ERR_SHAPE, "bias_act: bias has %lld entries for %lld planes",
                            nel(d->src[1]), dst.ne[2]);
            if (p[14] < 0 || p[14] > 2) return fail(PPDL_ERR_SHAPE, "bias_act: act %lld", p[14]);
            return to_status(ppdl::launch_bias_act((const float *)s0.data,
                                                   (const float *)d->src[1].data, (float *)dst.data, n,
                                                   dst.ne[0] * dst.ne[1], (int)dst.ne[2], p[14], st));
        }
        case PPDL_OP_COPY: {
            const long long n = nel(dst);
            if (nel(s0) < n) return fail(PPDL_ERR_SHAPE, "copy: src %lld < dst %lld", nel(s0), n);
            return to_status(ppdl::launch_copy((const float *)s0.data, (float *)dst.data, n, st));
        }
        case PPDL_OP_TOPK: {
            // patch:771-777: src0 ne(nc, ntok), dst i32 ne(nq); pages in ne[2] / ne[1]
            const long long nc = s0.ne[0], ntok = s0.ne[1], B = s0.ne[2] * s0.ne[3];
            const long long nq = dst.ne[0];
            if (dst.ne[1] * dst.ne[2] * dst.ne[3] != B)
                return fail(PPDL_ERR_SHAPE, "topk: %lld dst pages vs %lld src pages",
                            dst.ne[1] * dst.ne[2] * dst.ne[3], B);
            if (ntok > 16384 || nq > ntok)
                return fail(PPDL_ERR_SHAPE, "topk: ntok %lld (max 16384), nq %lld", ntok, nq);
            return to_status(ppdl::launch_topk((const float *)s0.data, (int32_t *)dst.data, (int)ntok,
                                               (int)nc, (int)nq, (int)B, st));
        }
        default: {
            int status = PPDL_ERR_UNSUPPORTED;
            if (ppdl::ops_ext_launch(d, st, &status, g_err, sizeof g_err)) return status;
            return fail(PPDL_ERR_UNSUPPORTED, "op id %lld is not provided by this build", p[13]);
        }
    }
}

}  // extern "C"
