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

// Metadata of the k - 1 chained draft passes that follow a verification, computed on the
// device from the step's acceptance so the whole speculative step replays as one CUDA graph.
// Sequence b held base[b] tokens before the step (0: a padding row of the graph batch) and
// accepted acc[b] drafts, so it now holds base + acc + 1 tokens; chain pass j (1 .. k-1)
// runs the MTP layer at position p = base + acc - 1 + j (the row that reads token p + 1 and
// predicts token p + 2), writes its KV at p and attends to p + 1 keys.
// Outputs are [k - 1][B] (row j - 1 for pass j); padding rows get slot -1 (no KV write).
__global__ void spec_chain_meta_kernel(const int* __restrict__ base, const int* __restrict__ acc,
                                       const int* __restrict__ block_table, int bt_stride, int max_blocks,
                                       int block_size, int B, int k, int* __restrict__ pos, int* __restrict__ slot,
                                       int* __restrict__ kv_len) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int n0 = base[b];
  const int a = n0 > 0 ? min(max(acc[b], 0), k) : 0;
  for (int j = 1; j < k; ++j) {
    const int o = (j - 1) * B + b;
    const int p = n0 + a - 1 + j;
    const int blk = p / block_size;
    if (n0 <= 0 || p < 0 || blk >= max_blocks) {
      pos[o] = 0;
      slot[o] = -1;
      kv_len[o] = 1;
      continue;
    }
    pos[o] = p;
    slot[o] = block_table[(size_t)b * bt_stride + blk] * block_size + p % block_size;
    kv_len[o] = p + 1;
  }
}

}  // namespace xtu

extern "C" int xtu_spec_chain_meta(const int* base, const int* acc, const int* block_table, int bt_stride,
                                   int max_blocks, int block_size, int B, int k, int* pos, int* slot, int* kv_len,
                                   cudaStream_t s) {
  if (B <= 0 || k <= 1) return 0;
  xtu::spec_chain_meta_kernel<<<(B + 127) / 128, 128, 0, s>>>(base, acc, block_table, bt_stride, max_blocks,
                                                               block_size, B, k, pos, slot, kv_len);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

extern "C" int xtu_spec_verify(const int* target, const int* ids, const int* q_start, int B, int k, int* accepted,
                               int* last_row, cudaStream_t s) {
  if (B <= 0) return 0;
  xtu::spec_verify_kernel<<<(B + 127) / 128, 128, 0, s>>>(target, ids, q_start, B, k, accepted, last_row);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}
