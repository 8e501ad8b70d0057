// hostcopy.h -- moving logits from HBM into host memory that the caller owns.
//
// The reference's host program receives its logits in a malloc'd buffer and
// frees it itself (src/gpt/gpt2_call.cpp:66-68, :93-94), so the drop-in entry
// point must write pageable memory.  A plain cudaMemcpy into pageable memory
// runs at a fraction of the PCIe rate (the driver stages it through one
// pinned buffer and one host thread).  Here the copy is a pipeline instead:
// DMA of the next chunks into pinned staging buffers while a pool of host
// threads copies the current chunk out (and takes the destination's first-
// touch page faults in parallel).  Pinned destinations take one strided DMA.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gpt2 {

// Host memory for `bytes` of output that the caller releases with free():
// 2 MiB-aligned and marked for transparent huge pages when large (fewer,
// cheaper first-touch faults), plain malloc otherwise.  nullptr on failure.
void *alloc_host_output(size_t bytes);

// Copies `rows` rows of `cols` floats from device memory (row stride ld
// floats) into host memory dst (row stride cols), after the work already
// enqueued on st, and returns when dst is complete.  0 or a negative
// GPT2_E* code (the error text is set).
int copy_rows_to_host(const float *d_src, int64_t ld, int64_t rows, int64_t cols, float *dst, cudaStream_t st);

// Frees the pinned staging buffers (the model's shutdown calls it).
void release_host_staging();

}  // namespace gpt2
