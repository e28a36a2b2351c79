/*
 * Exact sequential-fmaf BAG primitive: TEST INFRASTRUCTURE ONLY (an oracle).
 *
 * out(i,j) = sum_k (x(i,k) + delta*y(i,k)) * (v(k,j) + eps*w(k,j))
 *
 * evaluated as the chain acc = fmaf(left, right, acc) over k = 0..K-1 from
 * acc = 0, with each operand sum rounded once in FP32 before the product.
 * That is the per-element order of the reference's SIMT primitive
 * (include/bag/cuda/detail/simt.cuh:14-33 for the operand sums,
 * simt.cuh:136-159 for the fmaf chain), so a CUDA primitive that keeps this
 * order reproduces it bit for bit.  All matrices are column-major with the
 * given leading dimensions.  Built with -ffp-contract=off so the operand sums
 * are not fused into the fmaf.
 */
#include <math.h>
#include <stddef.h>

void oracle_primitive_exact(int m, int n, int k,
                            const float* x, const float* y, const float* v, const float* w,
                            int ldx, int ldy, int ldv, int ldw, int delta, int eps,
                            float* out, int ldo) {
    for (int j = 0; j < n; ++j) {
        for (int i = 0; i < m; ++i) {
            float acc = 0.0f;
            for (int kk = 0; kk < k; ++kk) {
                float left = x[i + (size_t)kk * ldx];
                if (delta) left = left + (float)delta * y[i + (size_t)kk * ldy];
                float right = v[kk + (size_t)j * ldv];
                if (eps) right = right + (float)eps * w[kk + (size_t)j * ldw];
                acc = fmaf(left, right, acc);
            }
            out[i + (size_t)j * ldo] = acc;
        }
    }
}
