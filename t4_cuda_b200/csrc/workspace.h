// Library-managed scratch memory for kernels that combine partial results
// across CTAs (the streaming GEMV's split-tile fix-up).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace t4b {

struct Workspace {
    unsigned* error;      // sticky device error word (bit 0: a bounded wait timed out)
    unsigned* counters;   // zero between launches: every kernel resets what it used
    float* part;          // partial sums, no initial value required
};

// Scratch for `stream` on the current device with room for `counter_words`
// counters and `part_floats` partial sums.  One buffer per (device, stream):
// kernels queued on the same stream run in order, so they can share it.  The
// buffer is allocated (cudaMalloc) and zeroed on the first request and grown
// when a request is larger, also while the stream is being captured into a
// CUDA graph (the allocation then happens at capture time, outside the graph);
// buffers are never freed.
int acquire_workspace(cudaStream_t stream, size_t counter_words, size_t part_floats, Workspace* ws);

}  // namespace t4b
