// zs_noalloc_scratch.cu -- the fixed device scratch behind zs_sample_noalloc.
//
// Kept in a translation unit of its own so that the array sits in a module of
// its own: under lazy module loading (CUDA_MODULE_LOADING=LAZY) a process that
// never calls zs_sample_noalloc never loads this module and never holds the
// memory.  With eager loading every process that loads the library holds it.
#include <cuda_runtime.h>

#include "zs_sampler.h"

static __device__ __align__(256) unsigned char zs_noalloc_scratch[ZS_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch on the current device (loads the module on
// first use).  Not exported: only zs_sample_noalloc calls it.
__attribute__((visibility("hidden"))) cudaError_t zs_noalloc_scratch_address(void** ptr) {
    return cudaGetSymbolAddress(ptr, zs_noalloc_scratch);
}
