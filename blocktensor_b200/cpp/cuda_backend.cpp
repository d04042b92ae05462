// cuda_backend.cpp -- see cuda_backend.hpp.
#include "cuda_backend.hpp"

#include <cstring>
#include <stdexcept>

#include "bt_cuda.h"

namespace blocktensor {

void bt_throw_if_error(int status, const char* what) {
    if (status == BT_OK) return;
    std::string msg = std::string(what) + ": " + bt_cuda_last_error();
    switch (status) {
        case BT_ERR_OUT_OF_RANGE: throw std::out_of_range(msg);
        case BT_ERR_INVALID_ARGUMENT: throw std::invalid_argument(msg);
        default: throw std::runtime_error(msg);
    }
}

// ---------------------------------------------------------------- CudaBuffer

CudaBuffer::CudaBuffer(int device, size_t bytes, DataType dt, BufferUsage usage, MemoryLocation location)
    : device_(device), bytes_(bytes), dt_(dt), usage_(usage), location_(location) {
    bt_throw_if_error(bt_cuda_alloc(device_, bytes_, &dev_), "CudaBuffer allocation");
}

CudaBuffer::~CudaBuffer() { bt_cuda_free(device_, dev_); }

void* CudaBuffer::map() {
    shadow_.resize(bytes_);
    bt_throw_if_error(bt_cuda_copy_d2h(device_, shadow_.data(), dev_, bytes_), "CudaBuffer::map");
    mapped_ = true;
    return shadow_.data();
}

void CudaBuffer::unmap() {
    if (!mapped_) return;
    bt_throw_if_error(bt_cuda_copy_h2d(device_, dev_, shadow_.data(), bytes_), "CudaBuffer::unmap");
    mapped_ = false;
    std::vector<uint8_t>().swap(shadow_);
}

void CudaBuffer::write(const void* src, size_t bytes, size_t offset) {
    if (offset + bytes > bytes_) throw std::runtime_error("CudaBuffer::write out of bounds");
    bt_throw_if_error(bt_cuda_copy_h2d(device_, static_cast<uint8_t*>(dev_) + offset, src, bytes), "CudaBuffer::write");
    if (mapped_) std::memcpy(shadow_.data() + offset, src, bytes);
}

void CudaBuffer::read(void* dst, size_t bytes, size_t offset) {
    if (offset + bytes > bytes_) throw std::runtime_error("CudaBuffer::read out of bounds");
    bt_throw_if_error(bt_cuda_copy_d2h(device_, dst, static_cast<const uint8_t*>(dev_) + offset, bytes),
                      "CudaBuffer::read");
}

// ---------------------------------------------------------------- CudaBackend

CudaBackend::CudaBackend(int device) : device_(device) {
    char name[256] = {0};
    uint64_t total = 0;
    uint32_t threads = 0, smem = 0;
    bt_throw_if_error(bt_cuda_device_info(device, name, &total, &threads, &smem), "CudaBackend");
    info_.name = name;
    info_.vendor_name = "NVIDIA";
    info_.vendor_id = 0x10DE;
    info_.is_discrete = true;
    info_.total_vram_bytes = total;
    info_.max_workgroup_size[0] = threads;
    info_.max_workgroup_size[1] = threads;
    info_.max_workgroup_size[2] = 64;
    info_.max_workgroup_invocations = threads;
    info_.max_shared_memory_bytes = smem;
}

std::shared_ptr<IComputeBuffer> CudaBackend::create_buffer(size_t bytes, DataType dt, BufferUsage usage,
                                                           MemoryLocation location) {
    return std::make_shared<CudaBuffer>(device_, bytes, dt, usage, location);
}

std::shared_ptr<IComputePipeline> CudaBackend::create_pipeline_from_spirv(const std::string& name,
                                                                          const std::vector<uint32_t>&, size_t,
                                                                          size_t) {
    return std::make_shared<CudaPipeline>(name);
}

static void* dptr(const std::shared_ptr<IComputeBuffer>& b, const char* what) {
    auto cb = std::dynamic_pointer_cast<CudaBuffer>(b);
    if (!cb) throw std::runtime_error(std::string("CudaBackend::dispatch non-CudaBuffer passed (") + what + ")");
    return cb->device_ptr();
}

void CudaBackend::dispatch(const std::shared_ptr<IComputePipeline>& pipeline,
                           const std::vector<std::shared_ptr<IComputeBuffer>>& buffers,
                           const DispatchDimensions& dims, const void* push, size_t push_size) {
    auto p = std::dynamic_pointer_cast<CudaPipeline>(pipeline);
    if (!p) throw std::runtime_error("CudaBackend::dispatch invalid pipeline type");
    const std::string& n = p->name();
    auto need = [&](size_t nbuf, size_t nbytes) {
        if (buffers.size() < nbuf) throw std::invalid_argument("CudaBackend::dispatch: too few buffers for " + n);
        if (!push || push_size < nbytes) throw std::invalid_argument("CudaBackend::dispatch: push constants for " + n);
    };
    uint32_t u[4] = {0, 0, 0, 0};
    if (n == "matvec_q8_0") {
        need(3, 8);
        std::memcpy(u, push, 8);
        bt_throw_if_error(bt_cuda_matvec_q8_0(dptr(buffers[0], "W"), static_cast<const float*>(dptr(buffers[1], "X")),
                                              static_cast<float*>(dptr(buffers[2], "Y")), u[0], u[1], nullptr),
                          "matvec_q8_0");
    } else if (n == "matvec_q4_0") {
        need(3, 8);
        std::memcpy(u, push, 8);
        bt_throw_if_error(bt_cuda_matvec_q4_0(dptr(buffers[0], "W"), static_cast<const float*>(dptr(buffers[1], "X")),
                                              static_cast<float*>(dptr(buffers[2], "Y")), u[0], u[1], nullptr),
                          "matvec_q4_0");
    } else if (n == "rmsnorm") {
        need(3, 8);
        float eps;
        std::memcpy(u, push, 4);
        std::memcpy(&eps, static_cast<const uint8_t*>(push) + 4, 4);
        bt_throw_if_error(bt_cuda_rmsnorm(static_cast<const float*>(dptr(buffers[0], "X")),
                                          static_cast<const float*>(dptr(buffers[1], "W")),
                                          static_cast<float*>(dptr(buffers[2], "Out")), dims.x, u[0], eps, nullptr),
                          "rmsnorm");
    } else if (n == "rope") {
        need(2, 16);
        std::memcpy(u, push, 16);
        // in place when both bindings are the same buffer (transformer_engine.cpp:127,131)
        bt_throw_if_error(bt_cuda_rope(static_cast<const float*>(dptr(buffers[0], "in")),
                                       static_cast<float*>(dptr(buffers[1], "out")), u[0], u[1], u[2], u[3], 10000.0f,
                                       nullptr),
                          "rope");
    } else if (n == "softmax") {
        need(2, 8);
        std::memcpy(u, push, 8);
        bt_throw_if_error(bt_cuda_softmax(static_cast<const float*>(dptr(buffers[0], "in")),
                                          static_cast<float*>(dptr(buffers[1], "out")), u[0], u[1], nullptr),
                          "softmax");
    } else if (n == "silu") {
        need(2, 4);
        std::memcpy(u, push, 4);
        bt_throw_if_error(bt_cuda_silu(static_cast<const float*>(dptr(buffers[0], "in")),
                                       static_cast<float*>(dptr(buffers[1], "out")), u[0], nullptr),
                          "silu");
    }
    // other names: no-op pipeline, as CPUBackend (cpu_backend.cpp:68-72)
}

void CudaBackend::synchronize() { bt_throw_if_error(bt_cuda_synchronize(device_), "synchronize"); }

}  // namespace blocktensor
