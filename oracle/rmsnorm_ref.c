/*
 * ORACLE -- test infrastructure only. Not part of the product.
 *
 * Plain-C restatement of the reference's own CPU reference loops
 * (rmsnorm/csrc/ptx_rmsnorm_kernels.cu:6619-6721, `reference_fwd` / `reference_bwd` of
 * Int21-AI/RMSNorm-H100): sequential fp32 accumulation with fmaf per row, per-head affine
 * row `row % H`, dweight/dbias accumulated over rows in row order. Inputs and outputs are
 * fp32 arrays; callers convert half/bf16 to fp32 before and round after.
 *
 * Built by oracle/build_oracle.py into oracle/_build/liboracle_c.so with -ffp-contract=off
 * so that only the fmaf calls below fuse. Used by tests/test_oracle_golden.py as a second,
 * independent restatement next to oracle/rmsnorm_oracle.py.
 */
#include <math.h>
#include <stdint.h>

/* ptx_rmsnorm_kernels.cu:6619-6667 */
void oracle_fwd(const float* x, const float* residual, const float* weight, const float* bias,
                int64_t rows, int64_t n, int64_t heads, float eps, float* y, float* h_out,
                float* rstd_out) {
  for (int64_t row = 0; row < rows; ++row) {
    const int64_t base = row * n;
    const int64_t abase = (heads > 1 ? row % heads : 0) * n;
    float sq = 0.0f;
    for (int64_t c = 0; c < n; ++c) {
      float v = x[base + c];
      if (residual) v += residual[base + c];
      sq = fmaf(v, v, sq);
    }
    const float rstd = 1.0f / sqrtf(sq / (float)n + eps);
    if (rstd_out) rstd_out[row] = rstd;
    for (int64_t c = 0; c < n; ++c) {
      float v = x[base + c];
      if (residual) v += residual[base + c];
      if (h_out) h_out[base + c] = v;
      float o = v * rstd;
      if (weight) o *= weight[abase + c];
      if (bias) o += bias[abase + c];
      y[base + c] = o;
    }
  }
}

/* ptx_rmsnorm_kernels.cu:6669-6721. dweight / dbias must be zeroed by the caller
 * (heads * n floats each) and are accumulated in row order. */
void oracle_bwd(const float* x, const float* weight, const float* dout, const float* dresidual_out,
                const float* rstd, int64_t rows, int64_t n, int64_t heads, float* dx,
                float* dweight, float* dbias) {
  for (int64_t row = 0; row < rows; ++row) {
    const int64_t base = row * n;
    const int64_t abase = (heads > 1 ? row % heads : 0) * n;
    const float r = rstd[row];
    float dot = 0.0f;
    for (int64_t c = 0; c < n; ++c) {
      const float xh = x[base + c] * r;
      float wdy = dout[base + c];
      if (weight) wdy *= weight[abase + c];
      dot = fmaf(xh, wdy, dot);
    }
    const float mean = dot / (float)n;
    for (int64_t c = 0; c < n; ++c) {
      const float dy = dout[base + c];
      const float xh = x[base + c] * r;
      float wdy = dy;
      if (weight) wdy *= weight[abase + c];
      float g = (wdy - xh * mean) * r;
      if (dresidual_out) g += dresidual_out[base + c];
      dx[base + c] = g;
      if (dweight) dweight[abase + c] += dy * xh;
      if (dbias) dbias[abase + c] += dy;
    }
  }
}
