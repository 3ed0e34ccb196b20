// dropin.cu -- the reference's kernel entry points over host pointers.
//
// k3_mxfp4_dequant, k3_matmul_mxfp4, k3_matmul_q8, k3_matmul, k3_matmul_bf16 and k3_router
// keep the reference's signatures (include/k3/k3.h:241-243, 281-285, 559-566; k3_matmul is
// declared at src/core/k3_ops.c:265) and contract: void return, output
// fully written on return, and a precondition violation aborts with a FATAL message
// rather than returning with the output unwritten (src/core/k3_ops.c:37-78, 1366-1384).
// Each call stages its inputs into a per-device workspace, runs the device kernel on a
// private stream, copies the result back and synchronises. A CUDA failure is fatal for
// the same reason an allocation failure is fatal in the reference.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

namespace k3c {
int launch_mx_gemv(float *y, int ldy, const float *x, int ldx, int ntok, const uint8_t *packed,
                   const uint8_t *scales, int in, int rows, int group, cudaStream_t s);
int launch_mx_dequant(float *out, const uint8_t *packed, const uint8_t *scales, int rows,
                      int pcols, int group, cudaStream_t s);
int launch_mx_exact(float *y, int ldy, const float *x, int ldx, int ntok, const uint8_t *packed,
                    const uint8_t *scales, int in, int rows, int group, cudaStream_t s);
int launch_q8_pack(int8_t *wq, float *wscale, int ldw, const void *rows, int in, int out,
                   cudaStream_t s);
int launch_q8_gemv(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok,
                   const int8_t *wq, const float *wscale, int ldw, int in, int out, cudaStream_t s);
int launch_router(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                  const float *bias, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                  int ntok, double *part, cudaStream_t s);
size_t router_scratch_bytes(int hidden, int n_experts, int ntok);
int launch_mmw(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int wdt, int in, int out,
               int accumulate, cudaStream_t s);

[[noreturn]] static void fatal(const char *what, const char *detail) {
    fprintf(stderr, "k3c: FATAL, %s: %s\n    Aborting rather than returning with the output "
                    "buffer unwritten.\n", what, detail);
    abort();
}

// One growable device buffer and one stream per device, shared by the drop-in calls.
struct Workspace {
    std::mutex mu;
    char *buf = nullptr;
    size_t cap = 0;
    cudaStream_t stream = nullptr;
};
static Workspace g_ws[16];

static Workspace &ws_for_current(const char *what) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) fatal(what, "no CUDA device");
    return g_ws[dev];
}

static char *ws_reserve(Workspace &w, size_t bytes, const char *what) {
    if (!w.stream && cudaStreamCreateWithFlags(&w.stream, cudaStreamNonBlocking) != cudaSuccess)
        fatal(what, "cudaStreamCreate failed");
    if (bytes > w.cap) {
        if (w.buf) cudaFree(w.buf);
        w.buf = nullptr;
        w.cap = 0;
        const size_t want = align_up(bytes, (size_t)1 << 20);
        if (cudaMalloc((void **)&w.buf, want) != cudaSuccess) fatal(what, "cudaMalloc of the staging workspace failed");
        w.cap = want;
    }
    return w.buf;
}

static void cuda_ok(cudaError_t e, const char *what) {
    if (e != cudaSuccess) fatal(what, cudaGetErrorString(e));
}
static void rc_ok(int rc, const char *what) {
    if (rc != K3C_OK) fatal(what, k3c_last_error());
}

}  // namespace k3c

using namespace k3c;

extern "C" {

long k3_expert_drops = 0;

void k3_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                      int rows, int pcols, int group) {
    const char *what = "k3_mxfp4_dequant";
    if (rows <= 0 || pcols <= 0) return;
    if (group <= 0) fatal(what, "group must be positive");
    const int ngrp = (2 * pcols + group - 1) / group;
    const size_t nb_p = (size_t)rows * pcols, nb_s = (size_t)rows * ngrp;
    const size_t nb_o = (size_t)rows * 2 * pcols * sizeof(float);
    Workspace &w = ws_for_current(what);
    std::lock_guard<std::mutex> lk(w.mu);
    const size_t o_p = 0, o_s = align_up(nb_p, 256), o_o = align_up(o_s + nb_s, 256);
    char *b = ws_reserve(w, o_o + nb_o, what);
    cuda_ok(cudaMemcpyAsync(b + o_p, packed, nb_p, cudaMemcpyHostToDevice, w.stream), what);
    cuda_ok(cudaMemcpyAsync(b + o_s, scales, nb_s, cudaMemcpyHostToDevice, w.stream), what);
    rc_ok(launch_mx_dequant((float *)(b + o_o), (const uint8_t *)(b + o_p),
                            (const uint8_t *)(b + o_s), rows, pcols, group, w.stream), what);
    cuda_ok(cudaMemcpyAsync(out, b + o_o, nb_o, cudaMemcpyDeviceToHost, w.stream), what);
    cuda_ok(cudaStreamSynchronize(w.stream), what);
}

void k3_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                     const unsigned char *scales, int in, int rows, int group) {
    const char *what = "k3_matmul_mxfp4";
    if (in & 1) {
        char d[96];
        snprintf(d, sizeof d, "in=%d is odd; packed rows are in/2 bytes", in);
        fatal(what, d);
    }
    if (group > 64) {
        char d[96];
        snprintf(d, sizeof d, "group=%d exceeds 64", group);
        fatal(what, d);
    }
    if (group <= 0) fatal(what, "group must be positive");
    if (rows <= 0 || in <= 0) return;
    const int ngrp = (in + group - 1) / group;
    const size_t nb_x = (size_t)in * sizeof(float), nb_p = (size_t)rows * (in / 2);
    const size_t nb_s = (size_t)rows * ngrp, nb_y = (size_t)rows * sizeof(float);
    Workspace &w = ws_for_current(what);
    std::lock_guard<std::mutex> lk(w.mu);
    const size_t o_x = 0, o_p = align_up(nb_x, 256), o_s = align_up(o_p + nb_p, 256);
    const size_t o_y = align_up(o_s + nb_s, 256);
    char *b = ws_reserve(w, o_y + nb_y, what);
    cuda_ok(cudaMemcpyAsync(b + o_x, x, nb_x, cudaMemcpyHostToDevice, w.stream), what);
    cuda_ok(cudaMemcpyAsync(b + o_p, packed, nb_p, cudaMemcpyHostToDevice, w.stream), what);
    cuda_ok(cudaMemcpyAsync(b + o_s, scales, nb_s, cudaMemcpyHostToDevice, w.stream), what);
    // the reference's own summation order: bit-identical for a group that is a multiple of 16
    rc_ok(launch_mx_exact((float *)(b + o_y), rows, (const float *)(b + o_x), in, 1,
                          (const uint8_t *)(b + o_p), (const uint8_t *)(b + o_s), in, rows, group,
                          w.stream), what);
    cuda_ok(cudaMemcpyAsync(y, b + o_y, nb_y, cudaMemcpyDeviceToHost, w.stream), what);
    cuda_ok(cudaStreamSynchronize(w.stream), what);
}

void k3_matmul_q8(float *y, const float *x, const void *W, int in, int out) {
    const char *what = "k3_matmul_q8";
    if (in <= 0 || out <= 0) return;
    const int ldw = (int)align_up((size_t)in, 32);
    const size_t nb_r = (size_t)out * (4 + (size_t)in), nb_x = (size_t)in * sizeof(float);
    const size_t nb_q = (size_t)out * ldw, nb_sc = (size_t)out * sizeof(float);
    const size_t nb_y = (size_t)out * sizeof(float);
    Workspace &w = ws_for_current(what);
    std::lock_guard<std::mutex> lk(w.mu);
    const size_t o_r = 0, o_x = align_up(nb_r, 256), o_q = align_up(o_x + nb_x, 256);
    const size_t o_sc = align_up(o_q + nb_q, 256), o_y = align_up(o_sc + nb_sc, 256);
    char *b = ws_reserve(w, o_y + nb_y, what);
    cuda_ok(cudaMemcpyAsync(b + o_r, W, nb_r, cudaMemcpyHostToDevice, w.stream), what);
    cuda_ok(cudaMemcpyAsync(b + o_x, x, nb_x, cudaMemcpyHostToDevice, w.stream), what);
    rc_ok(launch_q8_pack((int8_t *)(b + o_q), (float *)(b + o_sc), ldw, b + o_r, in, out, w.stream), what);
    rc_ok(launch_q8_gemv((float *)(b + o_y), out, b + o_x, K3C_F32, in, 1, (const int8_t *)(b + o_q),
                         (const float *)(b + o_sc), ldw, in, out, w.stream), what);
    cuda_ok(cudaMemcpyAsync(y, b + o_y, nb_y, cudaMemcpyDeviceToHost, w.stream), what);
    cuda_ok(cudaStreamSynchronize(w.stream), what);
}

static void trunk_matmul(float *y, const float *x, const void *W, int wdt, int in, int out, const char *what) {
    if (out <= 0) return;
    if (in <= 0) {   // an empty sum is zero
        memset(y, 0, (size_t)out * sizeof(float));
        return;
    }
    const size_t esz = wdt == K3C_WBF16 ? 2 : 4;
    const size_t nb_w = (size_t)out * in * esz, nb_x = (size_t)in * sizeof(float);
    const size_t nb_y = (size_t)out * sizeof(float);
    Workspace &w = ws_for_current(what);
    std::lock_guard<std::mutex> lk(w.mu);
    const size_t o_w = 0, o_x = align_up(nb_w, 256), o_y = align_up(o_x + nb_x, 256);
    char *b = ws_reserve(w, o_y + nb_y, what);
    cuda_ok(cudaMemcpyAsync(b + o_w, W, nb_w, cudaMemcpyHostToDevice, w.stream), what);
    cuda_ok(cudaMemcpyAsync(b + o_x, x, nb_x, cudaMemcpyHostToDevice, w.stream), what);
    rc_ok(launch_mmw((float *)(b + o_y), out, (const float *)(b + o_x), in, 1, b + o_w, wdt, in, out, 0, w.stream),
          what);
    cuda_ok(cudaMemcpyAsync(y, b + o_y, nb_y, cudaMemcpyDeviceToHost, w.stream), what);
    cuda_ok(cudaStreamSynchronize(w.stream), what);
}

void k3_matmul(float *y, const float *x, const float *W, int in, int out) {
    trunk_matmul(y, x, W, K3C_WF32, in, out, "k3_matmul");
}

void k3_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out) {
    trunk_matmul(y, x, W, K3C_WBF16, in, out, "k3_matmul_bf16");
}

void k3_router(int *idx, float *wout, const float *x, const float *W, const float *bias,
               int hidden, int n_experts, int topk, int renorm, float routed_scale) {
    const char *what = "k3_router";
    if (topk <= 0) return;
    if (n_experts <= 0 || hidden <= 0) fatal(what, "empty router");
    const size_t nb_x = (size_t)hidden * sizeof(float), nb_w = (size_t)n_experts * hidden * sizeof(float);
    const size_t nb_b = bias ? (size_t)n_experts * sizeof(float) : 0;
    const size_t nb_sc = router_scratch_bytes(hidden, n_experts, 1);   // logit chunks
    const size_t nb_i = (size_t)topk * sizeof(int), nb_o = (size_t)topk * sizeof(float);
    Workspace &w = ws_for_current(what);
    std::lock_guard<std::mutex> lk(w.mu);
    const size_t o_x = 0, o_w = align_up(nb_x, 256), o_b = align_up(o_w + nb_w, 256);
    const size_t o_sc = align_up(o_b + nb_b, 256), o_i = align_up(o_sc + nb_sc, 256);
    const size_t o_o = align_up(o_i + nb_i, 256);
    char *b = ws_reserve(w, o_o + nb_o, what);
    cuda_ok(cudaMemcpyAsync(b + o_x, x, nb_x, cudaMemcpyHostToDevice, w.stream), what);
    cuda_ok(cudaMemcpyAsync(b + o_w, W, nb_w, cudaMemcpyHostToDevice, w.stream), what);
    if (bias) cuda_ok(cudaMemcpyAsync(b + o_b, bias, nb_b, cudaMemcpyHostToDevice, w.stream), what);
    rc_ok(launch_router((int *)(b + o_i), (float *)(b + o_o), nullptr, b + o_x, K3C_F32, b + o_w, K3C_F32,
                        bias ? (const float *)(b + o_b) : nullptr, hidden, n_experts, topk, renorm, routed_scale,
                        1, (double *)(b + o_sc), w.stream), what);
    cuda_ok(cudaMemcpyAsync(idx, b + o_i, nb_i, cudaMemcpyDeviceToHost, w.stream), what);
    cuda_ok(cudaMemcpyAsync(wout, b + o_o, nb_o, cudaMemcpyDeviceToHost, w.stream), what);
    cuda_ok(cudaStreamSynchronize(w.stream), what);
}

}  // extern "C"
