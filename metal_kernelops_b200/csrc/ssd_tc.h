// Tensor-core (tcgen05) path of the Mamba-2 SSD chunk scan, called from the
// C-ABI entry points of mamba2_chunk.cu when eligible() holds.
#pragma once

#include <cuda_runtime.h>

#include "ssm_b200.h"

namespace ssm {
namespace ssdtc {

bool eligible(const ssm_chunk_scan_params* p);
void sizes(const ssm_chunk_scan_params* p, size_t* saved_bytes, size_t* workspace_bytes);
int fwd(const ssm_chunk_scan_params* p, cudaStream_t stream);
int bwd(const ssm_chunk_scan_params* p, cudaStream_t stream);

}  // namespace ssdtc
}  // namespace ssm
