// gdn_decode.cuh -- the kernel-sequence step's Gated DeltaNet decode layer.
//
// Value head h is split over kGdnSlices CTAs of 16 state rows each (grid
// values * kGdnSlices, kGdnThreads threads): the causal convolution and
// SiLU of the head's q, k and v channels, the L2 normalisation of q and k,
// the decay and beta gates, and the delta-rule update of the CTA's state
// rows (run_gdn's arithmetic, the same order as the dataflow step's GDN
// phase).  The output norm runs in the out-projection's prologue.
#pragma once

#include "common.cuh"
#include "model_kernels.cuh"

namespace prism {

constexpr int kGdnWarps = kGdnThreads / 32;
constexpr int kGdnSlices = 8;  // CTAs per value head: 16 state rows each

// Gated DeltaNet layer, value head h split over kGdnSlices CTAs of 16 state
// rows (arithmetic of gdn_decode_kernel; the output norm runs in the next
// projection's prologue).  o (pre-norm) goes to a.attended.
__device__ void run_gdn(const GdnArgs &a, int pos, uint8_t *scratch,
                        const float4 *preloaded = nullptr) {
  constexpr int S = 128, R = S / kGdnSlices;
  if ((int)blockIdx.x >= a.values * kGdnSlices) return;
  float *q = reinterpret_cast<float *>(scratch);  // [S]
  float *k = q + S;                              // [S]
  float *v = k + S;                              // [R]
  double *red = reinterpret_cast<double *>(v + R + 16);
  float *sdb = reinterpret_cast<float *>(red + kGdnWarps);  // decay, beta
  const int h = blockIdx.x / kGdnSlices, slice = blockIdx.x % kGdnSlices, r0 = slice * R;
  const int kh = h % a.groups, kw = a.groups * S, hist = a.conv_k - 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int parity = pos & 1;
  const float *hist_in = a.conv_state + parity * a.conv_buf_stride;
  float *hist_out = a.conv_state + (parity ^ 1) * a.conv_buf_stride;
  // 1. convolution + SiLU of the head's q, k channels and this slice's v
  if (tid < 2 * S + R) {
    const int part = tid < S ? 0 : tid < 2 * S ? 1 : 2;
    const int j = part < 2 ? tid - part * S : r0 + (tid - 2 * S);
    const int ch = part == 0 ? kh * S + j : part == 1 ? kw + kh * S + j : 2 * kw + h * S + j;
    const float projected = a.mixed[ch];
    const float *hj = hist_in + (long)ch * hist;
    const float *cj = a.conv_w + (long)ch * a.conv_k;
    float sum = 0.0f;
    for (int i = 0; i < hist; ++i) sum = __fadd_rn(sum, __fmul_rn(hj[i], cj[i]));
    sum = __fadd_rn(sum, __fmul_rn(projected, cj[hist]));
    const float act = silu_f(sum);
    if (part == 0) q[j] = act;
    else if (part == 1) k[j] = act;
    else v[j - r0] = act;
    if (part == 2 || (h == kh && slice == 0)) {
      float *nj = hist_out + (long)ch * hist;
      for (int i = 0; i + 1 < hist; ++i) nj[i] = hj[i + 1];
      if (hist > 0) nj[hist - 1] = projected;
    }
  }
  if (tid == 0) {
    sdb[0] = recurrent_decay_f(a.alpha_in[h], a.dt_bias[h], a.ssm_a[h], a.status);
    sdb[1] = sigmoid_f(a.beta_in[h]);
  }
  __syncthreads();
  // 2. L2 normalisation of q and k (same block-sum order as the kernel)
  {
    const float xq = tid < S ? q[tid] : 0.0f;
    const float xk = tid < S ? k[tid] : 0.0f;
    const double sq = block_sum_f64(tid < S ? (double)__fmul_rn(xq, xq) : 0.0, red);
    const double sk = block_sum_f64(tid < S ? (double)__fmul_rn(xk, xk) : 0.0, red);
    const float scq = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sq), a.eps));
    const float sck = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sk), a.eps));
    __syncthreads();
    if (tid < S) {
      q[tid] = __fmul_rn(xq, scq);
      k[tid] = __fmul_rn(xk, sck);
    }
  }
  __syncthreads();
  // 3. this slice's state rows, one per warp
  const float decay = sdb[0], beta = sdb[1];
  const float oscale = __fdiv_rn(1.0f, __fsqrt_rn((float)S));
  if (warp < R) {
    const int r = r0 + warp;
    const float4 kk = reinterpret_cast<const float4 *>(k)[lane];
    const float4 qq = reinterpret_cast<const float4 *>(q)[lane];
    float *row = a.state + (long)h * S * S + (long)r * S;
    float4 s = preloaded ? *preloaded : reinterpret_cast<const float4 *>(row)[lane];
    s.x = __fmul_rn(decay, s.x);
    s.y = __fmul_rn(decay, s.y);
    s.z = __fmul_rn(decay, s.z);
    s.w = __fmul_rn(decay, s.w);
    double dk = (double)__fmul_rn(s.x, kk.x) + (double)__fmul_rn(s.y, kk.y) +
                (double)__fmul_rn(s.z, kk.z) + (double)__fmul_rn(s.w, kk.w);
    dk = warp_sum_f64(dk);
    const float delta = __fmul_rn(__fsub_rn(v[warp], (float)dk), beta);
    s.x = __fadd_rn(s.x, __fmul_rn(delta, kk.x));
    s.y = __fadd_rn(s.y, __fmul_rn(delta, kk.y));
    s.z = __fadd_rn(s.z, __fmul_rn(delta, kk.z));
    s.w = __fadd_rn(s.w, __fmul_rn(delta, kk.w));
    const bool finite =
        is_finite_f(s.x) && is_finite_f(s.y) && is_finite_f(s.z) && is_finite_f(s.w);
    double dq = (double)__fmul_rn(s.x, qq.x) + (double)__fmul_rn(s.y, qq.y) +
                (double)__fmul_rn(s.z, qq.z) + (double)__fmul_rn(s.w, qq.w);
    dq = warp_sum_f64(dq);
    reinterpret_cast<float4 *>(row)[lane] = s;
    if (lane == 0) a.attended[h * S + r] = __fmul_rn((float)dq, oscale);
    if (!__all_sync(0xffffffffu, finite) && lane == 0) report(a.status, kStatusNonfinite);
  }
}

// The kernel-sequence step's Gated DeltaNet layer: value head h split over
// kGdnSlices CTAs of 16 state rows (grid values * kGdnSlices, kGdnThreads
// threads), run_gdn's arithmetic.  Pre-norm o goes to a.attended; the gated
// output norm runs in the out-projection's prologue (kProGated), for which
// each CTA replaces its 16 z values by SiLU(z) in place.  The state row was
// written by this layer's previous step: it is loaded before the grid
// dependency.
__global__ void __launch_bounds__(kGdnThreads) gdn_slices_kernel(GdnArgs a) {
  constexpr int S = 128, R = S / kGdnSlices;
  __shared__ __align__(16) uint8_t scratch[2048];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x / kGdnSlices, slice = blockIdx.x % kGdnSlices;
  trace_stamp(a.trace, 0);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (warp < R && h < a.values)
    s = reinterpret_cast<const float4 *>(a.state + (long)h * S * S +
                                         (long)(slice * R + warp) * S)[lane];
  grid_dependency_wait();
  trace_stamp(a.trace, 1);
  grid_dependents_launch();
  run_gdn(a, *a.position, scratch, &s);
  if (threadIdx.x < R && h < a.values) {
    float *z = const_cast<float *>(a.zgate) + (long)h * S + slice * R + threadIdx.x;
    *z = silu_f(*z);
  }
  trace_exit(a.trace);
}

}  // namespace prism
