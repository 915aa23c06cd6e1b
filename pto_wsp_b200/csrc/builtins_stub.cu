// Temporary launchers for kernels not yet written.
#include "device.hpp"
namespace ptowsp::dev {
cudaError_t launch_paged_decode(const TaskBatch&, int, int, int, void*, size_t, cudaStream_t) { return cudaErrorNotSupported; }
size_t paged_decode_scratch_bytes(const TaskBatch&, int) { return 0; }
cudaError_t launch_indexer_score(const TaskBatch&, int, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_topk_select(const TaskBatch&, int, void*, size_t, cudaStream_t) { return cudaErrorNotSupported; }
size_t topk_select_scratch_bytes(const TaskBatch&) { return 0; }
}
