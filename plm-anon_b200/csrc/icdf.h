// Argument block of the inverse-CDF verify decode (icdf.cu), the PTP scheme's decode.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace plm {

constexpr int kIcdfMaxVocab = 53248;  // 208 KB of float32 probabilities in shared memory
constexpr int kIcdfMaxTopK = 256;

struct IcdfArgs {
  const float* logits;     // [n_rows][ld] float32
  int64_t ld;
  const float* u;          // [n_rows] uniforms, or with u_base the request's uniform stream [u_len]
  int n_rows, vocab, top_k;
  int64_t* tokens;         // [n_rows]
  int32_t* ids_out;        // nullable [n_rows][top_k]
  float* edges_out;        // nullable [n_rows][top_k]
  const int64_t* u_base;   // nullable device scalar: row r reads u[*u_base + r]
  int64_t u_len;
  int* err;
};

int icdf_launch(const IcdfArgs& a, cudaStream_t stream, bool pdl);

}  // namespace plm
