// vc_noalloc.cu - decode attention for callers that cannot allocate device
// memory.
//
// Some embedders cannot call cudaMalloc at all: a host that hands this library
// a fixed device arena and forbids allocations after start-up (real-time audio
// pipelines that must not stall in the driver's allocator mid-stream), or code
// running where device allocation is disallowed.  This entry point runs the same
// split-K decode attention as vox_cuda_attention_decode_dev, but its scratch
// (the per-split partial results, the split tickets and the ring descriptor)
// is a file-scope __device__ array that exists from the moment the library is
// loaded on a GPU, so a call allocates nothing.
#include "voxtral_cuda.h"

#include "vc_common.cuh"
#include "vc_internal.h"


#include <mutex>

using namespace vc;

namespace {

// Layout of the static scratch, in floats:
//   [0, 16)                  ring descriptor (StreamSlot, <= 64 bytes)
//   [16, 24)                 split tickets (8 KV heads)
//   [32, 32 + kPartML)       per-split (max, sum) of the 32 query heads
//   [.., .. + kPartO)        per-split weighted V sums of the 32 query heads
constexpr size_t kSlotFloats = 16, kTicketOff = 16, kPartOff = 32;
constexpr size_t kPartML = (size_t)kDecHeads * kAttnSplits * 2;
constexpr size_t kPartO = (size_t)kDecHeads * kAttnSplits * kHeadDim;
constexpr size_t kScratchFloats = kPartOff + kPartML + kPartO;   // ~2.1 MB

static_assert(sizeof(StreamSlot) <= kSlotFloats * sizeof(float), "descriptor fits its slot");

// Every GPU that loads the library holds this array until the process exits.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

constexpr int kMaxDev = 16;
float *g_scratch_addr[kMaxDev] = {};
std::mutex g_mu;

}  // namespace

// Maximum attended keys: the scratch holds kAttnSplits splits of 64 keys.
#define VOX_NOALLOC_MAX_KEYS (kAttnSplits * 64)

extern "C" int vox_cuda_attention_decode_noalloc(const float *q, const float *k_ring,
                                                 const float *v_ring, int kv_cap, int pos,
                                                 float *out, void *stream) {
    if (!q || !k_ring || !v_ring || !out || kv_cap <= 0 || pos < 0) {
        vc::set_last_error("attention_decode_noalloc: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if ((((uintptr_t)q | (uintptr_t)k_ring | (uintptr_t)v_ring | (uintptr_t)out) & 15u) != 0) {
        vc::set_last_error("attention_decode_noalloc: pointers must be 16-byte aligned");
        return VOX_CUDA_ERR_ARG;
    }
    const int n_keys = (pos + 1 < kDecWindow) ? pos + 1 : kDecWindow;
    // With today's constants the window (8192) equals the scratch's capacity,
    // so this cannot fire; it guards a later change of either constant.
    if (n_keys > VOX_NOALLOC_MAX_KEYS) {
        vc::set_last_error("attention_decode_noalloc: %d keys exceed the static scratch (max %d)", n_keys,
                 VOX_NOALLOC_MAX_KEYS);
        return VOX_CUDA_ERR_CAPACITY;
    }
    if (n_keys > kv_cap) {
        vc::set_last_error("attention_decode_noalloc: ring of %d positions cannot hold %d keys", kv_cap, n_keys);
        return VOX_CUDA_ERR_CAPACITY;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
        vc::set_last_error("attention_decode_noalloc: no current device");
        return VOX_CUDA_ERR_UNAVAILABLE;
    }
    float *base;
    {
        // First call on a device: look up the array's device address with that
        // device current (the host-side symbol is not a device address).
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch_addr[dev]) {
            void *ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess || !ptr) {
                vc::set_last_error("attention_decode_noalloc: cudaGetSymbolAddress: %s",
                         cudaGetErrorString(e));
                return VOX_CUDA_ERR_CUDA;
            }
            g_scratch_addr[dev] = (float *)ptr;
        }
        base = g_scratch_addr[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    StreamSlot h = {const_cast<float *>(k_ring), const_cast<float *>(v_ring), kv_cap, pos,
                    pos % kv_cap, n_keys, pos};
    StreamSlot *slot = reinterpret_cast<StreamSlot *>(base);
    unsigned *tickets = reinterpret_cast<unsigned *>(base + kTicketOff);
    // the descriptor and the tickets (which must start at zero) are rewritten
    // by every call: the array keeps the previous call's contents.  A launch
    // that completes leaves its tickets at zero already; the reset is for a
    // previous launch that failed or was cut short, so it stays.
    if (cudaMemcpyAsync(slot, &h, sizeof(h), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemsetAsync(tickets, 0, kDecKvHeads * sizeof(unsigned), st) != cudaSuccess) {
        vc::set_last_error("attention_decode_noalloc: staging the descriptor failed");
        return VOX_CUDA_ERR_CUDA;
    }
    AttnParams p = {};
    p.q = q;
    p.slots = slot;
    p.layer = 0;
    p.out = out;
    p.part_ml = base + kPartOff;
    p.part_o = base + kPartOff + kPartML;
    p.counters = tickets;
    p.S = kAttnSplits;
    p.variant = 4;   // this entry keeps the v4 kernel its scratch was sized and tested for
    cudaError_t e = launch_attn_decode(1, p, st, false);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);   // h lives on this stack frame
    if (e != cudaSuccess) {
        vc::set_last_error("attention_decode_noalloc: %s", cudaGetErrorString(e));
        return VOX_CUDA_ERR_CUDA;
    }
    return VOX_CUDA_OK;
}
