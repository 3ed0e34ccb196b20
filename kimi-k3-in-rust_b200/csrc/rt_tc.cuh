// rt_tc.cuh -- shared between the tensor-core router logits (router_tc.cu) and the select
// kernel (router.cu): the digit split of a bf16 value and the residual lists the select
// kernel adds.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace k3c {

constexpr int RT_CAP = 64;              // residual entries kept per row
constexpr int RT_TC_MIN_TOKENS = 64;    // fewer tokens: the fp64 CUDA-core logits

// What the select kernel needs to finish the tensor-core logits of token t, expert e:
// the residual terms of token t's list (xk/xr[t*cap + i]) and of expert e's list
// (wk/wr[i*E + e]), or the whole double dot product when a list holds more than cap.
struct RtFix {
    const uint16_t *x, *W;   // bf16 [T][H] and [E][H]; x == nullptr: no tensor-core logits
    int H;
    const int *xexp, *xcnt, *xk;
    const float *xr;
    const int *wcnt, *wk;
    const float *wr;
    int cap;
};

__device__ __forceinline__ double rt_p2(int e) { return __longlong_as_double((long long)(e + 1023) << 52); }

// v on a row of exponent E (max|v| < 2^E) as 2^(E-6) (q0 + q1/128 + q2/128^2) + residual,
// |qj| <= 64; the residual is returned (exact in float).
__device__ __forceinline__ float rt_split(float v, int E, int &q0, int &q1, int &q2) {
    const float s = (float)((double)v * rt_p2(6 - E));   // |s| < 64: exact, or below the grid
    q0 = __float2int_rn(s);
    float r = s - (float)q0;
    q1 = __float2int_rn(r * 128.0f);
    r = r * 128.0f - (float)q1;
    q2 = __float2int_rn(r * 128.0f);
    const double rep = (double)(q0 * 16384 + q1 * 128 + q2) * rt_p2(E - 20);
    return (float)((double)v - rep);
}

bool router_tc_applies(int x_dtype, int w_dtype, int hidden, int ntok);
size_t router_tc_scratch_bytes(int hidden, int n_experts, int ntok);
int launch_router_tc(RtFix *fix, double **part, int *nslices, const void *x, const void *W, int hidden,
                     int n_experts, int ntok, void *scratch, cudaStream_t s);
int router_tc_check(cudaStream_t s);

}  // namespace k3c
