// Mamba-2 SSD chunk scan (placeholder until the kernels land).
#include "common.cuh"

using namespace ssm;

extern "C" int ssm_chunk_scan_sizes(const ssm_chunk_scan_params* p, size_t* saved_bytes,
                                    size_t* workspace_bytes) {
    if (saved_bytes) *saved_bytes = 0;
    if (workspace_bytes) *workspace_bytes = 0;
    return fail(SSM_ERR_UNSUPPORTED, "chunk_scan: not built yet");
}
extern "C" int ssm_chunk_scan_fwd(const ssm_chunk_scan_params* p, void* stream) {
    return fail(SSM_ERR_UNSUPPORTED, "chunk_scan: not built yet");
}
extern "C" int ssm_chunk_scan_bwd(const ssm_chunk_scan_params* p, void* stream) {
    return fail(SSM_ERR_UNSUPPORTED, "chunk_scan: not built yet");
}
