// Speculative-decoding verification (greedy): for each sequence, the number of
// leading draft tokens equal to the target model's greedy tokens, and the row of
// the last accepted position (whose hidden state seeds the next draft).
// Replaces the proposer/verifier that vLLM runs for the reference's MTP drafters
// (scripts/serve_v41.sh:41-47).
#include <cuda_runtime.h>

namespace xtu {

// one thread per sequence; rows q_start[b] .. q_start[b+1]-1 hold [last, d_1 .. d_n]
__global__ void spec_verify_kernel(const int* __restrict__ target, const int* __restrict__ ids,
                                   const int* __restrict__ q_start, int B, int k, int* __restrict__ accepted,
                                   int* __restrict__ last_row) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int q0 = q_start[b], q1 = q_start[b + 1];
  int a = 0;
  while (a < k && q0 + a + 1 < q1 && ids[q0 + a + 1] == target[q0 + a]) ++a;
  accepted[b] = a;
  last_row[b] = q0 + a;
}

}  // namespace xtu

extern "C" int xtu_spec_verify(const int* target, const int* ids, const int* q_start, int B, int k, int* accepted,
                               int* last_row, cudaStream_t s) {
  if (B <= 0) return 0;
  xtu::spec_verify_kernel<<<(B + 127) / 128, 128, 0, s>>>(target, ids, q_start, B, k, accepted, last_row);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}
