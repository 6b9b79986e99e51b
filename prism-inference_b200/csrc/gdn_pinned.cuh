// gdn_pinned.cuh -- the reference's pinned ("Swift") GDN recurrence on the
// device: every state row of every head stepped token by token in the
// arithmetic of src/kernels/pinned_gdn.rs (step_row_in_place :370-398 over
// tokens as step_row_tokens_from :401-455 and step_head_tokens_in_place
// :853-973 do; the scalar contract dot_scalar :205-230 and
// scalar_add_scaled :975-985, which the reference's NEON paths match bit for
// bit).  Per row and token:
//   row *= decay                       (separate binary32 multiplies)
//   dot_k = pinned dot(row, key)       (16 lanes: lane (4 reg + l) of each
//                                       16-element step accumulates by fused
//                                       multiply-add; registers 0+2 and 1+3,
//                                       then adjacent lane pairs)
//   delta = (value - dot_k) * beta     (separately rounded)
//   row += delta * key                 (fused over the 16-aligned prefix)
//   out = pinned dot(row, query) * (1 / sqrt(d))
// d = 128 (the device GDN width), so there is no unaligned tail.  A
// nonfinite dot or updated element reports nonfinite, where the reference
// returns its error.
//
// One CTA per (head, sequence) and a thread per state row, the row held in
// registers across the tokens (the loops over its 128 elements are unrolled);
// the token's key and query are staged in shared memory and read as float4
// broadcasts.
#pragma once

#include "common.cuh"
#include "gdn.cuh"

namespace prism {

constexpr int kPinnedD = 128;

__device__ __forceinline__ float pinned_tree(const float (&s)[4][4]) {
  float lanes[4];
#pragma unroll
  for (int l = 0; l < 4; ++l)
    lanes[l] = __fadd_rn(__fadd_rn(s[0][l], s[2][l]), __fadd_rn(s[1][l], s[3][l]));
  return __fadd_rn(__fadd_rn(lanes[0], lanes[1]), __fadd_rn(lanes[2], lanes[3]));
}

// grid (heads, batch), kPinnedD threads
__global__ void __launch_bounds__(kPinnedD, 1) gdn_pinned_kernel(GdnBatchArgs a) {
  constexpr int D = kPinnedD;
  __shared__ __align__(16) float kq[2][D];
  __shared__ float gb[2];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int kh = h % a.key_heads;
  grid_dependency_wait();
  grid_dependents_launch();
  float *srow = a.state + (((long)b * a.heads + h) * D + r) * D;
  float row[D];
#pragma unroll
  for (int x = 0; x < D / 4; ++x) {
    const float4 v4 = reinterpret_cast<const float4 *>(srow)[x];
    row[4 * x] = v4.x;
    row[4 * x + 1] = v4.y;
    row[4 * x + 2] = v4.z;
    row[4 * x + 3] = v4.w;
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
  bool finite = true;
  for (int t = 0; t < a.T; ++t) {
    const long tok = (long)b * a.T + t;
    __syncthreads();  // the previous token's key and query are no longer read
    kq[0][r] = a.k[(tok * a.key_heads + kh) * D + r];
    kq[1][r] = a.q[(tok * a.key_heads + kh) * D + r];
    if (r == 0) {
      gb[0] = a.decay[tok * a.heads + h];
      gb[1] = a.beta[tok * a.heads + h];
    }
    const float value = a.v[(tok * a.heads + h) * D + r];
    __syncthreads();
    const float decay = gb[0], beta = gb[1];
    float s[4][4];
#pragma unroll
    for (int g = 0; g < 4; ++g)
#pragma unroll
      for (int l = 0; l < 4; ++l) s[g][l] = 0.0f;
    // decay_and_dot: the row scaled, then its pinned dot with the key
#pragma unroll
    for (int x = 0; x < D / 4; ++x) {
      const float4 k4 = reinterpret_cast<const float4 *>(kq[0])[x];
      const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        row[4 * x + l] = __fmul_rn(row[4 * x + l], decay);
        s[x % 4][l] = fmaf(row[4 * x + l], kv[l], s[x % 4][l]);
      }
    }
    const float dot_k = pinned_tree(s);
    finite &= is_finite_f(dot_k);
    const float delta = __fmul_rn(__fsub_rn(value, dot_k), beta);
    // update_and_dot: the fused update, then the pinned dot with the query
#pragma unroll
    for (int g = 0; g < 4; ++g)
#pragma unroll
      for (int l = 0; l < 4; ++l) s[g][l] = 0.0f;
#pragma unroll
    for (int x = 0; x < D / 4; ++x) {
      const float4 k4 = reinterpret_cast<const float4 *>(kq[0])[x];
      const float4 q4 = reinterpret_cast<const float4 *>(kq[1])[x];
      const float kv[4] = {k4.x, k4.y, k4.z, k4.w}, qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const float e = fmaf(delta, kv[l], row[4 * x + l]);
        finite &= is_finite_f(e);
        row[4 * x + l] = e;
        s[x % 4][l] = fmaf(e, qv[l], s[x % 4][l]);
      }
    }
    const float dot_q = pinned_tree(s);
    finite &= is_finite_f(dot_q);
    a.out[(tok * a.heads + h) * D + r] = __fmul_rn(dot_q, scale);
  }
#pragma unroll
  for (int x = 0; x < D / 4; ++x)
    reinterpret_cast<float4 *>(srow)[x] =
        make_float4(row[4 * x], row[4 * x + 1], row[4 * x + 2], row[4 * x + 3]);
  if (!__syncthreads_and(finite) && r == 0) report(a.status, kStatusNonfinite);
}

}  // namespace prism
