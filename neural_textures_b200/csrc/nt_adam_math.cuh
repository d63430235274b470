// nt_adam_math.cuh -- the per-entry Adam update shared by the fused Adam launch and the
// sharded network update.
//
// AdamUpdateParameter (mavenkim2/neural_textures train.cu:521-543): the float operations are
// written out with explicit rounding in the order of the reference expression, so the result
// is bit-identical to the CPU oracle; the bias corrections 1 - beta^t come from the host.
#pragma once

namespace nt {

__device__ __forceinline__ float adam_update(float w, float g, float &m, float &v, float lr, float beta1, float beta2,
                                             float eps, float bc1, float bc2)
{
    const float m1 = __fadd_rn(__fmul_rn(beta1, m), __fmul_rn(__fsub_rn(1.f, beta1), g));
    const float m2 = __fadd_rn(__fmul_rn(beta2, v), __fmul_rn(__fmul_rn(__fsub_rn(1.f, beta2), g), g));
    m = m1;
    v = m2;
    const float mhat = __fdiv_rn(m1, bc1);
    const float vhat = __fdiv_rn(m2, bc2);
    return __fsub_rn(w, __fdiv_rn(__fmul_rn(lr, mhat), __fadd_rn(__fsqrt_rn(vhat), eps)));
}

}  // namespace nt
