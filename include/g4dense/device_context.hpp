// The device a model runs on: the B200 counterpart of the reference's VulkanContext
// (include/g4dense/vk_context.hpp), which the reference's ForwardRunner and DraftRuntime take as
// std::shared_ptr<VulkanContext>. Opaque: it names one CUDA device and, for tensor-parallel runs,
// this process's rank and the NCCL communicator shared by the ranks.
#pragma once
#include <cstdint>
#include <memory>

#define G4DENSE_CXX_API __attribute__((visibility("default")))

namespace g4dense {

class G4DENSE_CXX_API DeviceContext {
   public:
    // device: CUDA ordinal (-1 = the calling thread's current device). tp_size > 1 joins a
    // tensor-parallel group of tp_size processes with one NCCL unique id (128 bytes, from
    // nccl_unique_id() on rank 0, passed to every rank by the caller); the call blocks until every
    // rank has joined. Throws std::runtime_error on failure.
    static std::shared_ptr<DeviceContext> create(int device = -1, int tp_rank = 0, int tp_size = 1,
                                                 const void* nccl_unique_id = nullptr);
    // Fills 128 bytes with a fresh NCCL unique id (rank 0 of a tensor-parallel group).
    static void nccl_unique_id(void* out128);
    ~DeviceContext();
    DeviceContext(const DeviceContext&) = delete;
    DeviceContext& operator=(const DeviceContext&) = delete;

    int device() const;
    int tp_rank() const;
    int tp_size() const;
    void* nccl_comm() const;  // ncclComm_t, or null at tp_size 1

   private:
    DeviceContext();
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace g4dense
