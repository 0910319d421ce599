// NCCL calls through dlopen'ed entry points (nccl_dl.cpp). Throws std::runtime_error if NCCL cannot be loaded.
#pragma once
#include <cuda_runtime_api.h>
#include <nccl.h>

namespace mkb {

ncclResult_t dl_get_unique_id(ncclUniqueId* id);
ncclResult_t dl_comm_init_rank(ncclComm_t* comm, int nranks, ncclUniqueId id, int rank);
ncclResult_t dl_comm_destroy(ncclComm_t comm);
ncclResult_t dl_all_reduce(const void* send, void* recv, size_t count, ncclDataType_t type, ncclRedOp_t op,
                           ncclComm_t comm, cudaStream_t stream);
ncclResult_t dl_all_gather(const void* send, void* recv, size_t count, ncclDataType_t type, ncclComm_t comm,
                           cudaStream_t stream);
ncclResult_t dl_broadcast(const void* send, void* recv, size_t count, ncclDataType_t type, int root, ncclComm_t comm,
                          cudaStream_t stream);
ncclResult_t dl_group_start();
ncclResult_t dl_group_end();
const char* dl_error_string(ncclResult_t r);

}  // namespace mkb
