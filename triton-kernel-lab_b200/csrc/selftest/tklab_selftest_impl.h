// Internal declarations shared by the translation units of the test-only
// library libtklab_selftest.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace tk {

// Sets a kernel's dynamic shared-memory limit once per device (guarded by a
// mutex); `slot` distinguishes the kernels of this library.
int set_smem_attr_once(const void* kernel, int bytes, int slot);

int launch_umma_diag(const CUtensorMap* tm_a, const CUtensorMap* tm_b, const uint32_t* a_words, float* c,
                     int mode, int n, bool bf16, unsigned long long timeout_ns, int* status,
                     cudaStream_t stream);

int launch_exp2_fma_pair(const float* x, float* y, int64_t n, cudaStream_t stream);

}  // namespace tk
