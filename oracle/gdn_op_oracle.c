/*
 * gdn_op_oracle.c -- the reference's batched gated-delta op with snapshots
 * and replay (src/backend/gdn.rs:24-300 CpuBackend::delta_values, operations
 * 100 and 101), restated on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY: never linked into the product library.
 *
 * Tensors are in ggml order ([ne0, ne1, ne2, ne3], ne0 fastest):
 *   q [width, q_heads, tokens, q_sequences], k [width, k_heads, tokens,
 *   k_sequences] (head h reads q/k head h % q_heads / k_heads, sequence s
 *   reads sequence s / (sequences / q_sequences)), v [width, heads, tokens,
 *   sequences], gate [gate_width (1 or width), heads, tokens, sequences],
 *   beta [1, heads, tokens, sequences], state table [width*width*heads,
 *   state_rows] (row r of head h at r*width*width*heads + h*width*width).
 * Per (sequence, head), tokens in order, state S[row][col]:
 *   raw gates: beta = 1/(1+exp(-beta)); gate = 0 when weight[h] == 0 (with
 *   finite gate and bias), else weight[h] * softplus(gate + bias[h])
 *   (softplus(x) = x above 20, else ln(1 + exp(x)));
 *   S[row][col] *= exp(gate[col]) (per-column gates) or exp(gate);
 *   delta[row] = (v[row] - dot(S_row, k)) * beta;
 *   S[row][col] += k[col] * delta[row];
 *   out[row] = dot(S_row, q) * (1/sqrt(width)),
 * with dot(a, b) = binary32(sum over columns in order of binary64 a*b).
 * Outputs: the attention rows, then (operation 100) `snapshots` states, slot
 * t' = tokens-1-token holding the state after `token` (slot 0 the final
 * state), or (operation 101, replay) the state after token tokens-depth and
 * depth-1 records per sequence (delta[heads*width], keys[heads*width],
 * decay[heads]) of the tokens after it, where depth = min(tokens,
 * snapshots).  Replay first re-applies `count` records of bank `bank`
 * (control[2s], control[2s+1]) to the loaded state; records are
 * [sequences][record_banks][record_bank_elems] (the reference's record tensor
 * shape [bank elements, banks, sequences]).  Raw gates with replay are
 * refused: the reference reads both from its eighth source tensor.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "prism_oracle.h"

static float op_dot(const float *a, const float *b, int n) {
  double s = 0.0;
  for (int i = 0; i < n; ++i) s += (double)a[i] * (double)b[i];
  return (float)s;
}

int po_gdn_delta_values(const po_gdn_op *op, const float *q, const float *k, const float *v,
                        const float *gate, const float *beta, const float *table,
                        const int32_t *rows, const float *bias, const float *weight,
                        const float *records, const int32_t *control, float *out) {
  const int W = (int)op->width, H = (int)op->heads, T = (int)op->tokens, S = (int)op->sequences;
  const int snaps = (int)op->snapshots, replay = op->replay != 0;
  if (snaps == 0 || (replay && snaps < 2) || (replay && op->raw)) return PO_E_INVALID;
  if (W == 0 || H == 0 || S == 0 || (replay && T == 0) || op->q_sequences == 0 ||
      op->k_sequences == 0 || S % (int)op->q_sequences || S % (int)op->k_sequences ||
      (op->gate_width != 1 && op->gate_width != op->width))
    return PO_E_INVALID;
  const size_t per_head = (size_t)W * W, per_seq = per_head * H, all_state = per_seq * S;
  const size_t attn = (size_t)W * H * T * S;
  const size_t rec_w = (size_t)(2 * W + 1) * H;
  /* the state rows of the table each sequence reads (distinct, in range) */
  int *srow = (int *)malloc(sizeof(int) * (size_t)S);
  if (!srow) return PO_E_INVALID;
  for (int s = 0; s < S; ++s) {
    srow[s] = s;
    if (!replay && rows) {
      if (rows[s] < 0 || (uint32_t)rows[s] >= op->state_rows) {
        free(srow);
        return PO_E_INVALID;
      }
      for (int t = 0; t < s; ++t)
        if (rows[t] == rows[s]) {
          free(srow);
          return PO_E_INVALID;
        }
      srow[s] = rows[s];
    } else if ((uint32_t)s >= op->state_rows) {
      free(srow);
      return PO_E_INVALID;
    }
  }
  const int depth = T < snaps ? T : snaps;
  const int base = replay ? T - depth : 0;
  const float scale = 1.0f / sqrtf((float)W);
  float *st = (float *)malloc(sizeof(float) * per_head);
  float *delta = (float *)malloc(sizeof(float) * (size_t)W);
  if (!st || !delta) {
    free(srow);
    free(st);
    free(delta);
    return PO_E_INVALID;
  }
  int status = PO_OK;
  const int qs = S / (int)op->q_sequences, ks = S / (int)op->k_sequences;
  for (int s = 0; s < S && !status; ++s) {
    for (int h = 0; h < H && !status; ++h) {
      memcpy(st, table + (size_t)srow[s] * per_seq + (size_t)h * per_head, per_head * 4);
      if (replay) {
        const int count = control[2 * s], bank = control[2 * s + 1];
        if (count < 0 || count >= snaps || bank < 0 || bank > 1) {
          status = PO_E_INVALID;
          break;
        }
        /* records [sequence][banks][bank elements]; a bank holds records of
         * rec_w values each, the first `count` of them applied in order */
        const size_t rbase =
            ((size_t)s * op->record_banks + (size_t)bank) * op->record_bank_elems;
        if (bank >= (int)op->record_banks || rbase + (size_t)count * rec_w > op->records_len) {
          status = PO_E_INVALID;
          break;
        }
        for (int r = 0; r < count; ++r) {
          const float *rec = records + rbase + (size_t)r * rec_w;
          const float d = rec[2 * H * W + h];
          for (size_t x = 0; x < per_head; ++x) st[x] *= d;
          const float *kk = rec + (size_t)H * W + (size_t)h * W;
          for (int row = 0; row < W; ++row) {
            const float dl = rec[(size_t)h * W + row];
            for (int col = 0; col < W; ++col) st[(size_t)row * W + col] += kk[col] * dl;
          }
        }
      }
      for (int t = 0; t < T; ++t) {
        const float *qq = q + (((size_t)(s / qs) * T + t) * op->q_heads + h % op->q_heads) * W;
        const float *kk = k + (((size_t)(s / ks) * T + t) * op->k_heads + h % op->k_heads) * W;
        const float *vv = v + (((size_t)s * T + t) * H + h) * W;
        const size_t gi = ((size_t)s * T + t) * H + h;
        float bt = beta[gi];
        float g = gate[gi * op->gate_width];
        if (op->raw) {
          bt = 1.0f / (1.0f + po_expf(-bt));
          if (weight[h] == 0.0f && isfinite(g) && isfinite(bias[h])) {
            g = 0.0f;
          } else {
            const float x = g + bias[h];
            const float sp = x > 20.0f ? x : po_logf(1.0f + po_expf(x));
            g = weight[h] * sp;
          }
        }
        const float decay = po_expf(g);
        for (int row = 0; row < W; ++row)
          for (int col = 0; col < W; ++col) {
            const float f =
                op->gate_width == op->width ? po_expf(gate[gi * op->gate_width + col]) : decay;
            st[(size_t)row * W + col] *= f;
          }
        for (int row = 0; row < W; ++row)
          delta[row] = (vv[row] - op_dot(st + (size_t)row * W, kk, W)) * bt;
        for (int row = 0; row < W; ++row)
          for (int col = 0; col < W; ++col) st[(size_t)row * W + col] += kk[col] * delta[row];
        for (int row = 0; row < W; ++row)
          out[(((size_t)s * T + t) * H + h) * W + row] =
              op_dot(st + (size_t)row * W, qq, W) * scale;
        if (replay) {
          if (t == base) {
            memcpy(out + attn + (size_t)s * per_seq + (size_t)h * per_head, st, per_head * 4);
          } else if (t > base) {
            float *o = out + attn + all_state + ((size_t)s * (snaps - 1) + (t - base - 1)) * rec_w;
            memcpy(o + (size_t)h * W, delta, (size_t)W * 4);
            memcpy(o + (size_t)H * W + (size_t)h * W, kk, (size_t)W * 4);
            o[2 * (size_t)H * W + h] = decay;
          }
        } else {
          const int slot = T - 1 - t;
          if (slot < snaps)
            memcpy(out + attn + (size_t)slot * all_state + (size_t)s * per_seq +
                       (size_t)h * per_head,
                   st, per_head * 4);
        }
      }
      if (!replay && snaps == 1 && T == 0)
        memcpy(out + attn + (size_t)s * per_seq + (size_t)h * per_head, st, per_head * 4);
    }
  }
  free(srow);
  free(st);
  free(delta);
  return status;
}

size_t po_gdn_delta_values_outputs(const po_gdn_op *op) {
  const size_t W = op->width, H = op->heads, T = op->tokens, S = op->sequences;
  const size_t all_state = W * W * H * S, attn = W * H * T * S;
  if (op->replay)
    return attn + all_state + (size_t)(op->snapshots - 1) * (2 * W + 1) * H * S;
  return attn + (size_t)op->snapshots * all_state;
}
