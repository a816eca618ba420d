// Tensor-parallel collectives (NCCL loaded at run time; tp.cpp).
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

#include <string>

namespace myos {

bool tp_unique_id(uint8_t out[128], std::string* why);
bool tp_comm_init(ncclComm_t* comm, int size, int rank, const uint8_t id[128], std::string* why);
void tp_comm_destroy(ncclComm_t comm);
bool tp_allreduce_sum(const float* in, float* out, size_t n, ncclComm_t comm, cudaStream_t st);
bool tp_allgather(const void* in, void* out, size_t bytes, ncclComm_t comm, cudaStream_t st);

}  // namespace myos
