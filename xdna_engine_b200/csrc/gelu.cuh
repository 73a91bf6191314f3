// gelu.cuh -- the encoder GELU shared by every epilogue that applies it (the tcgen05 GEMM and
// the fused FFN), so the fused and unfused paths round identically.
//
// The reference's GELU: 0.5 x (1 + erf(x / sqrt 2)) with the Abramowitz-Stegun 7.1.26 erf,
// erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2), t = 1 / (1 + p z)
// (rust/npu-asr-host/src/lib.rs:464-495).  1 / (1 + p z) is the hardware approximate reciprocal
// (relative error below 2^-22, far under the formula's own 1.5e-7 absolute error), which has
// no slow path, so the unrolled epilogue loops interleave many independent evaluations.
#pragma once

namespace xdna {

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float gelu_erf_as(float v) {
    const float x = v * 0.70710678118654752440f;
    const float ax = fabsf(x);
    const float t = rcp_approx(fmaf(0.3275911f, ax, 1.0f));
    float p = fmaf(1.061405429f, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    const float y = fmaf(-p * t, __expf(-ax * ax), 1.0f);
    return 0.5f * v * (1.0f + copysignf(y, x));
}

}  // namespace xdna
