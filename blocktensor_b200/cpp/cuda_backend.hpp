// cuda_backend.hpp -- blocktensor::CudaBackend, the B200 implementation of the
// reference's IComputeBackend (runtime/include/blocktensor/backend.hpp:69-92).
//
// Drop-in location in the reference tree: backends/cuda/.  Plain C++ over the
// C ABI of libbt_cuda.so (include/bt_cuda.h); no CUDA headers needed.
//
// * CudaBuffer: device memory with the IComputeBuffer contract of CPUBuffer
//   (backends/cpu/cpu_backend.cpp:20-34): bounds-checked read/write that
//   throw std::runtime_error; map() returns a host shadow that unmap() writes
//   back (the staging path of memory/memory_manager.cpp:22-65 relies on it).
// * Pipelines are looked up by name and the SPIR-V is ignored, as
//   CPUBackend::create_pipeline_from_spirv does (cpu_backend.cpp:59-73).
//   Known names and push-constant layouts are those the engine binds
//   (runtime/src/transformer_engine.cpp:56-64,76,103,124,202):
//     "matvec_q8_0" {u32 M, N}            buffers {W, X, Y},   dims.x = M
//     "rmsnorm"     {u32 dim; f32 eps}    buffers {X, W, Out}, dims.x = rows
//     "rope"        {u32 seq, heads, hd, pos} buffers {in, out}
//     "softmax"     {u32 rows, dim}       buffers {in, out}
//     "silu"        {u32 n}               buffers {in, out}
//   Unknown names get a no-op pipeline, the CPUBackend behaviour.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "blocktensor/backend.hpp"

namespace blocktensor {

class CudaBuffer : public IComputeBuffer {
public:
    CudaBuffer(int device, size_t bytes, DataType dt, BufferUsage usage, MemoryLocation location);
    ~CudaBuffer() override;
    CudaBuffer(const CudaBuffer&) = delete;
    CudaBuffer& operator=(const CudaBuffer&) = delete;

    size_t size() const override { return bytes_; }
    DataType data_type() const override { return dt_; }
    BufferUsage usage() const override { return usage_; }
    MemoryLocation location() const override { return location_; }

    void* map() override;
    void unmap() override;
    void write(const void* src, size_t bytes, size_t offset = 0) override;
    void read(void* dst, size_t bytes, size_t offset = 0) override;

    void* device_ptr() const { return dev_; }
    int device() const { return device_; }

private:
    int device_;
    size_t bytes_;
    DataType dt_;
    BufferUsage usage_;
    MemoryLocation location_;
    void* dev_ = nullptr;
    std::vector<uint8_t> shadow_;
    bool mapped_ = false;
};

class CudaPipeline : public IComputePipeline {
public:
    explicit CudaPipeline(std::string name) : name_(std::move(name)) {}
    const std::string& name() const override { return name_; }

private:
    std::string name_;
};

class CudaBackend : public IComputeBackend {
public:
    explicit CudaBackend(int device = 0);
    ~CudaBackend() override = default;

    std::string backend_name() const override { return "CUDA_B200"; }
    const DeviceInfo& device_info() const override { return info_; }
    int device() const { return device_; }

    std::shared_ptr<IComputeBuffer> create_buffer(size_t bytes, DataType dt, BufferUsage usage,
                                                  MemoryLocation location) override;

    std::shared_ptr<IComputePipeline> create_pipeline_from_spirv(const std::string& name,
                                                                 const std::vector<uint32_t>& spirv_code,
                                                                 size_t buffer_binding_count,
                                                                 size_t push_constant_size = 0) override;

    void dispatch(const std::shared_ptr<IComputePipeline>& pipeline,
                  const std::vector<std::shared_ptr<IComputeBuffer>>& buffers, const DispatchDimensions& dims,
                  const void* push_constants = nullptr, size_t push_constants_size = 0) override;

    void synchronize() override;

private:
    int device_;
    DeviceInfo info_;
};

// Rethrows a bt_cuda status code as the exception type the reference uses.
void bt_throw_if_error(int status, const char* what);

}  // namespace blocktensor
