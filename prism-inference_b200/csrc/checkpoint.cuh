// checkpoint.cuh -- decoder checkpoints on the device (the reference's
// Decoder::checkpoint / checkpoint_into / restore / checkpoint_bytes,
// src/lib.rs:105,305-319, implemented for Qwen35 at src/graph.rs:5483-5578).
//
// A checkpoint is one device allocation holding every piece of decoder state
// a later step reads, in layer order:
//   full-attention layer: its K rows then its V rows of positions [0, p);
//   GDN layer:            its recurrent matrix, then both halves of its
//                         convolution history (the step's parity selects one);
// then the token history [0, p] (the next step's input included) and the
// prompt end.  Position 0 holds no layer payload, as in the reference.
// Copies run device to device on the model's stream.
#pragma once

#include "model.cuh"

struct prism_b200_checkpoint {
  uint64_t owner = 0;     // the model's serial (the reference's provenance)
  int device = 0;
  int64_t position = 0;
  uint8_t *data = nullptr;
  size_t bytes = 0, capacity = 0;
};

namespace prism {

// One piece of model state: device address and bytes at `position`.
struct StatePiece {
  void *ptr;
  size_t bytes;
};

inline std::vector<StatePiece> checkpoint_pieces(prism_b200_model *m, int64_t position) {
  const auto &c = m->cfg;
  std::vector<StatePiece> out;
  if (position > 0) {
    for (auto &Ly : m->L) {
      if (Ly.full) {
        out.push_back({Ly.kc, (size_t)position * m->kv_row_bytes()});
        out.push_back({Ly.vc, (size_t)position * m->kv_row_bytes(true)});
      } else {
        out.push_back({Ly.matrix, (size_t)c.ssm_values * c.ssm_state * c.ssm_state * 4});
        out.push_back({Ly.conv_state, (size_t)2 * m->channels() * (c.conv_kernel - 1) * 4});
      }
    }
  }
  out.push_back({m->d_tokens, (size_t)(position + 1) * 4});
  out.push_back({m->d_prompt_end, 4});
  return out;
}

inline size_t checkpoint_size(const std::vector<StatePiece> &ps) {
  size_t n = 0;
  for (const auto &p : ps) n += (p.bytes + 255) / 256 * 256;
  return n;
}

inline int checkpoint_fill(prism_b200_model *m, prism_b200_checkpoint *cp) {
  prism_b200_executor *ex = m->ex;
  const auto ps = checkpoint_pieces(m, m->position);
  const size_t need = checkpoint_size(ps);
  cudaSetDevice(ex->device);
  CK(cudaStreamSynchronize(m->stream), "model stream");
  if (need > cp->capacity) {
    if (cp->data) cudaFree(cp->data);
    cp->data = nullptr;
    cp->capacity = 0;
    CK(cudaMalloc(&cp->data, need), "checkpoint allocation");
    cp->capacity = need;
  }
  size_t off = 0;
  for (const auto &p : ps) {
    CK(cudaMemcpyAsync(cp->data + off, p.ptr, p.bytes, cudaMemcpyDeviceToDevice, m->stream),
       "checkpoint copy");
    off += (p.bytes + 255) / 256 * 256;
  }
  CK(cudaStreamSynchronize(m->stream), "checkpoint copy");
  cp->owner = m->serial;
  cp->device = ex->device;
  cp->position = m->position;
  cp->bytes = need;
  return PRISM_B200_OK;
}

}  // namespace prism

extern "C" {

int prism_b200_model_checkpoint(prism_b200_model *m, prism_b200_checkpoint **out) {
  if (!m || !out) return PRISM_B200_E_INVALID;
  *out = nullptr;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  auto *cp = new prism_b200_checkpoint();
  if ((st = prism::checkpoint_fill(m, cp))) {
    if (cp->data) cudaFree(cp->data);
    delete cp;
    return st;
  }
  *out = cp;
  return PRISM_B200_OK;
}

int prism_b200_model_checkpoint_into(prism_b200_model *m, prism_b200_checkpoint *cp) {
  if (!m || !cp) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (cp->data && cp->device != ex->device)
    return ex->fail(PRISM_B200_E_INVALID, "checkpoint storage lives on another device");
  return prism::checkpoint_fill(m, cp);
}

int prism_b200_model_restore(prism_b200_model *m, const prism_b200_checkpoint *cp) {
  using namespace prism;
  if (!m || !cp) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (cp->owner != m->serial || cp->device != ex->device || cp->position < 0 ||
      cp->position > (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID, "checkpoint belongs to a different model or context");
  if (cp->position == 0) return prism_b200_model_reset(m);
  const auto ps = checkpoint_pieces(m, cp->position);
  if (checkpoint_size(ps) != cp->bytes)
    return ex->fail(PRISM_B200_E_INVALID, "checkpoint belongs to a different model or context");
  cudaSetDevice(ex->device);
  size_t off = 0;
  for (const auto &p : ps) {
    CK(cudaMemcpyAsync(p.ptr, cp->data + off, p.bytes, cudaMemcpyDeviceToDevice, m->stream),
       "restore copy");
    off += (p.bytes + 255) / 256 * 256;
  }
  const int pos = (int)cp->position;
  CK(cudaMemcpyAsync(m->d_position, &pos, 4, cudaMemcpyHostToDevice, m->stream), "restore");
  CK(cudaStreamSynchronize(m->stream), "restore");
  m->position = cp->position;
  return PRISM_B200_OK;
}

int64_t prism_b200_checkpoint_bytes(const prism_b200_checkpoint *cp) {
  return cp ? (int64_t)cp->bytes : -1;
}

int64_t prism_b200_checkpoint_position(const prism_b200_checkpoint *cp) {
  return cp ? cp->position : -1;
}

void prism_b200_checkpoint_destroy(prism_b200_checkpoint *cp) {
  if (!cp) return;
  if (cp->data) {
    cudaSetDevice(cp->device);
    cudaFree(cp->data);
  }
  delete cp;
}

}  // extern "C"
