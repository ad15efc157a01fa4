// Greedy argmax over the rows of a logits matrix that needs no caller-provided
// workspace and allocates no device memory.  It has no counterpart in the
// reference, whose sampling is done by the serving framework around it.
//
// Defined in elementwise.cu beside the allocating entry point xtu_argmax.
#pragma once
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest number of rows one call accepts: the partial results of every row live
// in a fixed 512 KiB device array (1024 rows x 64 parts x 8 bytes).
#define XTU_ARGMAX_STATIC_MAX_ROWS 1024

// Return codes below -10000 are this entry point's own argument errors; other
// negative values are -(cudaError_t) of the failing CUDA call.
#define XTU_ARGMAX_STATIC_ERR_TOO_MANY_ROWS (-10001)
#define XTU_ARGMAX_STATIC_ERR_BAD_SIZE (-10002)
#define XTU_ARGMAX_STATIC_ERR_DEVICE (-10003)

// out[r] = lowest index of the largest value in row r of `logits` (fp32, or bf16 when
// is_bf16 != 0; row r starts at logits + r * stride elements), out_val[r] = that value
// (out_val may be NULL), for r < T.  Returns the number of kernels launched (1 or 2),
// 0 when T == 0, or a negative error code.
int xtu_argmax_static(const void* logits, int is_bf16, int T, int V, int stride, int* out, float* out_val,
                      cudaStream_t stream);

#ifdef __cplusplus
}
#endif
