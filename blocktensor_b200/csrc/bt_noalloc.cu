// bt_noalloc.cu -- the tile-layout GEMV for callers that cannot allocate.
//
// bt_cuda_gemv_q8_units takes the scratch it needs for row tiles split
// between CTAs (partial sums, arrival tickets, a timeout flag) from a
// per-device workspace that it cudaMallocs on first use.  Some callers cannot
// allow that: an engine that reserves all device memory up front in its own
// pool, a host runtime whose allocator must see every byte, or code that must
// not hit the allocator's implicit device synchronisation in its decode loop.
// bt_cuda_gemv_q8_units_noalloc runs the same kernel with that scratch in a
// fixed file-scope device array instead.
//
// The array is a static __device__ symbol, so every GPU that loads this
// library holds it (288 KB) until the process exits.  Host code must never
// pass the symbol itself to a kernel: on the host its name is only a stand-in,
// not a device address.  The device address is looked up once per device with
// cudaGetSymbolAddress, on the first call made with that device current.
#include "bt_common.cuh"
#include "bt_gemv_mma.cuh"
#include "bt_internal.h"

#include <mutex>

namespace bt {
namespace {

constexpr uint32_t kNoAllocMaxSMs = 256;                       // CTAs of one launch
constexpr uint32_t kNoAllocMaxRows = 1u << 20;                 // M
constexpr uint32_t kNoAllocPartFloats = kNoAllocMaxSMs * 256;  // partial sums
constexpr uint32_t kNoAllocTickets = 8192;                     // arrival tickets
// [partials][tickets][timeout flag], 256-byte aligned sections
constexpr size_t kNoAllocPartBytes = (size_t)kNoAllocPartFloats * sizeof(float);
constexpr size_t kNoAllocTicketBytes = (size_t)(kNoAllocTickets + 64) * sizeof(uint32_t);
constexpr size_t kNoAllocBytes = kNoAllocPartBytes + kNoAllocTicketBytes;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

struct NoAllocDevice {
    bool ready = false;
    unsigned char* base = nullptr;  // device address of g_noalloc_scratch on this device
    uint32_t nsm = 0;
};

std::mutex g_noalloc_mutex;
NoAllocDevice g_noalloc[64];

// Looks up the device address of the scratch array on the current device
// (once per device).  Allocates nothing.
int noalloc_setup(int dev, NoAllocDevice** out) {
    if (dev < 0 || dev >= 64) return fail(BT_ERR_INVALID_ARGUMENT, "gemv_q8_units_noalloc: device index above 63");
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocDevice& d = g_noalloc[dev];
    if (!d.ready) {
        int nsm = 0;
        BT_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
        if (nsm <= 0 || (uint32_t)nsm > kNoAllocMaxSMs)
            return fail(BT_ERR_INVALID_ARGUMENT,
                        "gemv_q8_units_noalloc: device has more SMs than the fixed scratch covers");
        void* p = nullptr;
        BT_CUDA_CHECK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        d.base = static_cast<unsigned char*>(p);
        d.nsm = (uint32_t)nsm;
        d.ready = true;
    }
    *out = &d;
    return BT_OK;
}

}  // namespace

int noalloc_inject_timeout(int device) {
    NoAllocDevice* d = nullptr;
    int rc = noalloc_setup(device, &d);  // the caller has made `device` current
    if (rc != BT_OK) return rc;
    const uint32_t one = 1;
    BT_CUDA_CHECK(cudaMemcpy(d->base + kNoAllocPartBytes + kNoAllocTickets * sizeof(uint32_t), &one, sizeof(one),
                             cudaMemcpyHostToDevice));
    return BT_OK;
}

}  // namespace bt

using namespace bt;

extern "C" int bt_cuda_gemv_q8_units_noalloc(const void* units, const float* x, float* y, uint32_t M, uint32_t K,
                                             void* stream) {
    BT_CHECK_ARG(K % 32 == 0 && K > 0, "gemv_q8_units_noalloc: K must be a positive multiple of 32");
    BT_CHECK_ARG(K <= kGemvMaxK, "gemv_q8_units_noalloc: K above 48384 not supported");
    BT_CHECK_ARG(M <= kNoAllocMaxRows, "gemv_q8_units_noalloc: M above 1048576 rows exceeds the fixed scratch");
    BT_CHECK_ARG(units && x && y, "gemv_q8_units_noalloc: null buffer");
    BT_CHECK_ARG(((uintptr_t)units & 15) == 0 && ((uintptr_t)x & 15) == 0,
                 "gemv_q8_units_noalloc: units and x must be 16-byte aligned");
    if (M == 0) return BT_OK;
    int dev = 0;
    BT_CUDA_CHECK(cudaGetDevice(&dev));
    NoAllocDevice* d = nullptr;
    int rc = noalloc_setup(dev, &d);
    if (rc != BT_OK) return rc;
    float* part = reinterpret_cast<float*>(d->base);
    uint32_t* ticket = reinterpret_cast<uint32_t*>(d->base + kNoAllocPartBytes);
    uint32_t* err = ticket + kNoAllocTickets;
    cudaStream_t s = as_stream(stream);
    // the tickets start at zero on every call; the partial sums need no clearing.  The
    // timeout flag is read (and cleared when set) after the call.
    BT_CUDA_CHECK(cudaMemsetAsync(ticket, 0, sizeof(uint32_t) * kNoAllocTickets, s));
    const UnitW w{static_cast<const uint8_t*>(units), M, unit_rows(M), K};
    BT_CUDA_CHECK(launch_gemv_mma(w, MProCopy{x}, SEpiStore{y}, SplitScratch{part, ticket}, err, d->nsm, s, false));
    return gemv_check_timeout(err, ticket, sizeof(uint32_t) * kNoAllocTickets, s);
}
