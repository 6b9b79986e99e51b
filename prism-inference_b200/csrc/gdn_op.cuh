// gdn_op.cuh -- the reference's batched gated-delta op with snapshots and
// replay (src/backend/gdn.rs:24-300 CpuBackend::delta_values, operations 100
// and 101) on the device.
//
// One CTA per (head, sequence), a thread per state row, the head's state in
// shared memory (rows padded by one word).  Per token, in order: every row's
// elements scaled by exp(gate) (or by exp(gate[col]) for per-column gates),
// delta = (v - dot(S_row, k)) * beta, S_row += k * delta, out = dot(S_row, q)
// * (1/sqrt(width)); dot = binary64 sum in column order of exact products,
// rounded to binary32; every binary32 operation unfused, as the reference's.
// Raw gates first map beta through the sigmoid and the gate through
// weight * softplus(gate + bias) (0 when weight is 0 with finite inputs).
// Outputs as the reference lays them out: the attention rows, then the
// snapshot slots (slot tokens-1-t holds the state after token t), or, in
// replay, the state after token tokens-depth and the later tokens' records
// (delta rows, keys, decay).  Replay first re-applies `count` records of the
// chosen bank to the loaded state.
#pragma once

#include "common.cuh"

namespace prism {

constexpr int kGdnOpMaxWidth = 128;

struct GdnOpArgs {
  int W, H, T, S, qh, kh, qs, ks, gw, snaps, raw, replay, state_rows, banks;
  long bank_elems, records_len;
  const float *q, *k, *v, *gate, *beta, *table;
  const int32_t *rows;
  const float *bias, *weight, *records;
  const int32_t *control;
  float *out;
  unsigned *status;
};

__host__ __device__ inline size_t gdn_op_outputs(long W, long H, long T, long S, long snaps,
                                                  bool replay) {
  const size_t all_state = (size_t)W * W * H * S, attn = (size_t)W * H * T * S;
  return replay ? attn + all_state + (size_t)(snaps - 1) * (2 * W + 1) * H * S
                : attn + (size_t)snaps * all_state;
}

__global__ void __launch_bounds__(kGdnOpMaxWidth) gdn_op_kernel(GdnOpArgs a) {
  extern __shared__ __align__(16) float gop_sm[];
  const int W = a.W, WP = W + 1, H = a.H, T = a.T, S = a.S;
  float *st = gop_sm;              // [W][W + 1]
  float *kq = st + W * WP;         // k[W], q[W]
  float *fac = kq + 2 * W;         // per-column factors [W]
  __shared__ float s_beta, s_decay;
  __shared__ int s_bad;
  const int h = blockIdx.x, s = blockIdx.y, row = threadIdx.x;
  const bool live = row < W;
  grid_dependency_wait();
  grid_dependents_launch();
  if (row == 0) s_bad = 0;
  __syncthreads();
  // the state row this sequence reads: distinct, inside the table
  int srow = s;
  if (!a.replay && a.rows) {
    srow = a.rows[s];
    bool bad = srow < 0 || srow >= a.state_rows;
    for (int t = row; t < s && !bad; t += blockDim.x) bad = a.rows[t] == srow;
    if (bad) atomicOr(&s_bad, 1);
  } else if (s >= a.state_rows) {
    if (row == 0) s_bad = 1;
  }
  __syncthreads();
  if (s_bad) {
    if (row == 0) report(a.status, kStatusInvalid);
    return;
  }
  const size_t per_head = (size_t)W * W, per_seq = per_head * H, all_state = per_seq * S;
  const size_t attn = (size_t)W * H * T * S, rec_w = (size_t)(2 * W + 1) * H;
  const float *src = a.table + (size_t)srow * per_seq + (size_t)h * per_head;
  for (int i = threadIdx.x; i < W * W; i += blockDim.x) st[(i / W) * WP + i % W] = src[i];
  if (a.replay) {
    const int count = a.control[2 * s], bank = a.control[2 * s + 1];
    const size_t rbase = ((size_t)s * a.banks + (size_t)(bank < 0 ? 0 : bank)) * a.bank_elems;
    if (count < 0 || count >= a.snaps || bank < 0 || bank > 1 || bank >= a.banks ||
        rbase + (size_t)count * rec_w > (size_t)a.records_len) {
      if (row == 0) report(a.status, kStatusInvalid);
      return;
    }
    __syncthreads();
    for (int r = 0; r < count; ++r) {
      const float *rec = a.records + rbase + (size_t)r * rec_w;
      if (live) {
        const float d = rec[2 * (size_t)H * W + h];
        const float dl = rec[(size_t)h * W + row];
        const float *kk = rec + (size_t)H * W + (size_t)h * W;
        float *sr = st + row * WP;
        for (int c = 0; c < W; ++c) sr[c] = __fmul_rn(sr[c], d);
        for (int c = 0; c < W; ++c) sr[c] = __fadd_rn(sr[c], __fmul_rn(kk[c], dl));
      }
    }
  }
  const int depth = T < a.snaps ? T : a.snaps;
  const int base = a.replay ? T - depth : 0;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)W));
  const int qsq = S / a.qs, ksq = S / a.ks;
  for (int t = 0; t < T; ++t) {
    __syncthreads();  // the previous token's k and q are no longer read
    const float *qq = a.q + (((size_t)(s / qsq) * T + t) * a.qh + h % a.qh) * W;
    const float *kk = a.k + (((size_t)(s / ksq) * T + t) * a.kh + h % a.kh) * W;
    const size_t gi = ((size_t)s * T + t) * H + h;
    if (live) {
      kq[row] = kk[row];
      kq[W + row] = qq[row];
      if (a.gw == W) fac[row] = exp_cr(a.gate[gi * a.gw + row]);
    }
    if (row == 0) {
      float bt = a.beta[gi], g = a.gate[gi * a.gw];
      if (a.raw) {
        bt = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-bt)));
        if (a.weight[h] == 0.0f && is_finite_f(g) && is_finite_f(a.bias[h])) {
          g = 0.0f;
        } else {
          const float x = __fadd_rn(g, a.bias[h]);
          const float sp = x > 20.0f ? x : log_cr(__fadd_rn(1.0f, exp_cr(x)));
          g = __fmul_rn(a.weight[h], sp);
        }
      }
      s_beta = bt;
      s_decay = exp_cr(g);
    }
    __syncthreads();
    if (!live) continue;
    float *sr = st + row * WP;
    const float decay = s_decay;
    double dk = 0.0;
    for (int c = 0; c < W; ++c) {
      const float x = __fmul_rn(sr[c], a.gw == W ? fac[c] : decay);
      sr[c] = x;
      dk = __fma_rn((double)x, (double)kq[c], dk);
    }
    const float vr = a.v[(((size_t)s * T + t) * H + h) * W + row];
    const float delta = __fmul_rn(__fsub_rn(vr, __double2float_rn(dk)), s_beta);
    double dq = 0.0;
    for (int c = 0; c < W; ++c) {
      const float x = __fadd_rn(sr[c], __fmul_rn(kq[c], delta));
      sr[c] = x;
      dq = __fma_rn((double)x, (double)kq[W + c], dq);
    }
    a.out[(((size_t)s * T + t) * H + h) * W + row] = __fmul_rn(__double2float_rn(dq), scale);
    if (a.replay) {
      if (t == base) {
        float *o = a.out + attn + (size_t)s * per_seq + (size_t)h * per_head + (size_t)row * W;
        for (int c = 0; c < W; ++c) o[c] = sr[c];
      } else if (t > base) {
        float *o = a.out + attn + all_state + ((size_t)s * (a.snaps - 1) + (t - base - 1)) * rec_w;
        o[(size_t)h * W + row] = delta;
        o[(size_t)H * W + (size_t)h * W + row] = kq[row];
        if (row == 0) o[2 * (size_t)H * W + h] = decay;
      }
    } else if (T - 1 - t < a.snaps) {
      float *o = a.out + attn + (size_t)(T - 1 - t) * all_state + (size_t)s * per_seq +
                 (size_t)h * per_head + (size_t)row * W;
      for (int c = 0; c < W; ++c) o[c] = sr[c];
    }
  }
  __syncthreads();  // with no tokens, the loaded state is read here
  if (!a.replay && a.snaps == 1 && T == 0 && live) {
    float *o = a.out + attn + (size_t)s * per_seq + (size_t)h * per_head + (size_t)row * W;
    for (int c = 0; c < W; ++c) o[c] = st[row * WP + c];
  }
}

}  // namespace prism
