// Allocation-free entry point for callers that cannot allocate device memory.
//
// This entry point has no counterpart in the reference project. It exists for
// hosts that must not call cudaMalloc/cudaFree (or any allocating library) on
// their own schedule -- for example a host that owns a fixed device-memory
// budget, or runs the kernel from a context where a driver allocation could
// block or fail -- yet still want this library's RMSNorm backward. The
// regular entry point obtains its scratch from torch's caching allocator;
// this one keeps it in a fixed device array instead.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// Widest rows served: 4096 columns for bf16, 2048 for fp32 (the fp32 dx
// kernel keeps a row in registers, 4 floats per 16-byte vector). Wider rows
// are rejected with error 2 before anything launches.
#define TS_NOALLOC_RMS_MAX_COLS_BF16 4096
#define TS_NOALLOC_RMS_MAX_COLS_FP32 2048
#define TS_NOALLOC_RMS_MAX_CHUNKS 128

// RMSNorm backward without allocating anything.
//   dy, x, dx : [rows, cols] row-major, bf16 (dtype 0) or fp32 (dtype 1)
//   w         : [cols], same dtype as x
//   rstd      : [rows] fp32, the forward's reciprocal RMS
//   dw        : [cols] fp32 output (overwritten, not accumulated)
//   stream    : the cudaStream_t to launch on
// dy, x, w and dx must be 16-byte aligned; rstd and dw 4-byte aligned.
// Returns 0 on success, or a nonzero code whose text ts_noalloc_last_error()
// returns: 1 bad argument (null or misaligned pointer, bad shape or dtype),
// 2 row width beyond the limit above, 4 no device / symbol lookup failed,
// 5 a launch of this call failed, 6 a CUDA error from earlier work was
// already pending (nothing was launched). Codes 1, 2 and 6 launch nothing.
int ts_rms_norm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                            int rows, int cols, int dtype, void* stream);

// Text of the calling thread's last error from the entry point above.
const char* ts_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
