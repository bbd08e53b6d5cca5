// thork_internal.h — declarations shared by the host-side translation units of
// libthork_rt.so (not part of the public C-ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

int thork_set_error(int code, const char *fmt, ...);
int thork_cuda_error(cudaError_t e, const char *what);
int thork_encode_tmap_2d(void *out128, int dtype, const void *base, uint64_t rows, uint64_t cols,
                         uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols,
                         int swizzle_bytes);
// Per-device status word (4 x u32, cudaMalloc'd and zeroed on first use).
int thork_status_word(unsigned **d_status);
// Cached multiprocessor count of the current device.
int thork_sm_count(int *n);
// Pipelined copies through pinned slots for pageable host memory (staging.cu).
bool thork_is_pageable(const void *host_ptr);
size_t thork_staged_min_bytes();
int thork_staged_htod(void *d_dst, const void *h_src, size_t n, cudaStream_t s);
int thork_staged_dtoh(void *h_dst, const void *d_src, size_t n, cudaStream_t s);
