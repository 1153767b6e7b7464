// error_word.cuh — the caller's error word, shared by the attention, linear
// and softmax kernels.
//
// A caller passes one int32 per launch (b200_*_params::error_word).  It may
// live in device memory, where kernels OR their error bits into it
// atomically, or in pinned host memory that the device addresses directly
// (cudaHostAlloc / torch pin_memory under unified addressing).  A host word
// can be read by the host at any time without synchronising, so each entry
// point reads it before launching and refuses to launch while an earlier
// launch's report is still in it.
//
// Inside the kernels a host word is marked by bit 0 of its address (the word
// is 4-byte aligned, so the bit is otherwise zero).  Kernels cannot rely on
// atomics over the host link, so they write a host word with a plain
// read-or-write followed by a system fence: two CTAs reporting at once may
// keep only one CTA's bits, but the word is never left zero by a report.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "b200_attn.h"

namespace b200attn {

__device__ __forceinline__ void report_error(int32_t* tagged, int32_t bits) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(tagged);
  if (!a) return;
  if (a & 1u) {
    volatile int32_t* w = reinterpret_cast<volatile int32_t*>(a & ~static_cast<uintptr_t>(1));
    *w = *w | bits;
    __threadfence_system();
  } else {
    atomicOr(tagged, bits);
  }
}

// Records the text b200_attn_last_error_detail returns (attn_fwd_sm100.cu).
void set_error(const char* msg);

// Resolves the caller's error word for a launch: `*kernel_word` receives the
// pointer the kernel gets (NULL, the device word, or the device address of a
// host word with bit 0 set).  A host word that already holds a report makes
// the call fail with B200_ATTN_ERR_TIMEOUT (the timeout bit) or
// B200_ATTN_ERR_DEVICE_BOUNDS (any other bit) before anything is launched.
inline int32_t resolve_error_word(int32_t* user, int32_t** kernel_word) {
  *kernel_word = nullptr;
  if (!user) return B200_ATTN_OK;
  if (reinterpret_cast<uintptr_t>(user) & 3u) {
    set_error("error_word is not 4-byte aligned");
    return B200_ATTN_ERR_ALIGNMENT;
  }
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, user) != cudaSuccess) {
    cudaGetLastError();
    set_error("error_word: cudaPointerGetAttributes failed");
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  }
  if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
    *kernel_word = user;
    return B200_ATTN_OK;
  }
  if (attr.type != cudaMemoryTypeHost || !attr.devicePointer) {
    set_error("error_word is host memory the device cannot address (not pinned and mapped)");
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  }
  const int32_t seen = *reinterpret_cast<volatile int32_t*>(user);
  if (seen != 0) {
    set_error("an earlier launch reported a device error in this error word; clear it to continue");
    return (seen & B200_ATTN_DEVERR_WAIT_TIMEOUT) ? B200_ATTN_ERR_TIMEOUT
                                                  : B200_ATTN_ERR_DEVICE_BOUNDS;
  }
  *kernel_word = reinterpret_cast<int32_t*>(reinterpret_cast<uintptr_t>(attr.devicePointer) | 1u);
  return B200_ATTN_OK;
}

// Counts one kernel launch of this library (b200_attn_launch_count).
void count_launch();

}  // namespace b200attn
