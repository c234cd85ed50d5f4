// select_noalloc.cu -- ugbsa_select for callers that cannot allocate device memory.
//
// ugbsa_select needs a small scratch area (per-tile sigma margins, per-tile head
// sums and means, the quantile threshold) that its caller passes in.  Some
// callers have no way to provide it: an inference server whose memory planner
// has already handed the whole device to a pool it manages, a host-language
// binding that only holds the input/output tensors given to it and no
// allocator, or code that must not call cudaMalloc because it would
// synchronise the device in the middle of a pipelined launch sequence.  For
// them, ugbsa_select_noalloc runs exactly the same kernels with the scratch
// taken from the fixed array below instead.
//
// Properties of that array:
//  * file-scope, statically sized at UGBSA_NOALLOC_SCRATCH_BYTES (1 MiB): every
//    GPU that loads libugbsa holds these bytes until the process exits;
//  * a call is accepted when the scratch ugbsa_select would lay out for it,
//    ugbsa_select_workspace_bytes_ex(cfg, dtype, B, Hq, Hkv, S, D), fits in it,
//    and refused with UGBSA_ERR_TOO_LARGE otherwise.  With bf16 Q and head_dim
//    64, 128 or 256 (the tensor-core scorer) that scratch holds the exact tile
//    scores, 4 * B * Hq * ceil(S/64)^2 bytes, which grows with the square of the
//    sequence: 28 query / 4 KV heads at head_dim 128 fit up to about 5K tokens,
//    one head up to about 28K.  Other dtypes and head dims need only about
//    4 * B * (Hq + 2) * ceil(S/64) bytes (28 heads: any S the selector accepts);
//  * shared by every call on a device and never cleared: each call writes every
//    scratch element it later reads, so nothing has to start at zero, but two
//    calls whose kernels overlap on the GPU (different streams, no ordering)
//    race on it;
//  * host code cannot use the array's name as a device address; its address is
//    looked up once per device with cudaGetSymbolAddress, with that device
//    current, on the first call of this entry point on that device.  That first
//    call should therefore be made before any stream capture begins.
#include <mutex>

#include "common.cuh"
#include "ugbsa_internal.h"

#define UGBSA_NOALLOC_SCRATCH_BYTES (1u << 20)

static __device__ __align__(256) unsigned char g_noalloc_scratch[UGBSA_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void *g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_address(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return UGBSA_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return UGBSA_ERR_NO_DEVICE;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return UGBSA_OK;
}

}  // namespace

extern "C" int ugbsa_select_noalloc(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a,
                                    const float *summ_b, int B, int Hq, int Hkv, int S, int D, float scale,
                                    const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma,
                                    uint8_t *trigger, ugbsa_stream_t stream) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0) return UGBSA_ERR_SHAPE;
    const size_t need = ugbsa::select_workspace_bytes_exact(dtype, B, Hq, Hkv, S, D);
    if (need > UGBSA_NOALLOC_SCRATCH_BYTES) return UGBSA_ERR_TOO_LARGE;
    void *scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc != UGBSA_OK) return rc;
    // same validation and kernels as ugbsa_select, with the fixed scratch as workspace
    return ugbsa_select(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, scale, cfg, kv_idx, kmax, sigma, trigger,
                        scratch, UGBSA_NOALLOC_SCRATCH_BYTES, stream);
}
