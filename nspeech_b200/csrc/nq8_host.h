// nq8_host.h -- host-side weight preparation (internal header).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "nq8_layout.h"

struct nq_weight;  // include/nq8.h

namespace nq {

constexpr int kPackGlu = 1;
constexpr int kErrIo = -8;
constexpr int kErrFormat = -7;

// Record `msg` as the calling thread's last error (nq_last_error) and return code.
int api_fail(int code, const std::string &msg);

// Kernel launches one nq_linear call of M rows makes on the current device
// (`aligned`: bf16 activations 16-byte aligned with ldx % 8 == 0).
int linear_launches(const ::nq_weight *w, int64_t m, int x_dtype, bool aligned);

int pack_n_tiles(int64_t n, int flags);
int pack_k_chunks(int64_t k);
// GGUF Q8_0 blocks [n][k/32] x 34 B  <->  tiles [n_tiles][kc] x 8704 B.
void pack_q8_0(const uint8_t *blocks, int64_t n, int64_t k, int flags, uint8_t *out);
void unpack_q8_0(const uint8_t *packed, int64_t n, int64_t k, int flags, uint8_t *blocks);
// f32 [n][k] -> bf16 (round to nearest even) rows in packed row order,
// [n_tiles * 128][kc * 64], zero past n and k: the layout of a kept bf16 copy.
void pack_bf16_rows(const float *w, int64_t n, int64_t k, int flags, uint16_t *out);
// f32 [n][k] -> GGUF Q8_0 blocks (ggml quantize_row_q8_0_ref semantics).
void quantize_q8_0(const float *w, int64_t n, int64_t k, uint8_t *blocks);
// First element of w[0, count) whose Q8_0 block does not dequantize back to
// it exactly (NaN never does), or -1.
int64_t q8_0_first_mismatch(const float *w, const uint8_t *blocks, int64_t count);

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;  // ne[0] (innermost) first
  uint32_t type = 0;           // ggml type id; Q8_0 = 8
  uint64_t offset = 0;         // relative to the data section
};

class GgufFile {
 public:
  ~GgufFile();
  int open(const char *path, std::string *err);  // 0 or kErr*
  const GgufTensor *find(const char *name) const;
  // Pointer to `bytes` bytes of tensor data, or null if out of the file.
  const uint8_t *data(const GgufTensor &t, size_t bytes) const;
  const std::vector<GgufTensor> &tensors() const { return tensors_; }

 private:
  int fd_ = -1;
  void *map_ = nullptr;
  size_t size_ = 0;
  size_t data_start_ = 0;
  std::vector<GgufTensor> tensors_;
};

}  // namespace nq
