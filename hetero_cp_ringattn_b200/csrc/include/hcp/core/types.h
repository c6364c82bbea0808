// Language-neutral core types: tensor descriptors, ring / domain configuration.
//
// Parity: include/hcp_ringattn/core/tensor_types.h:7-27 (BoundaryTensor) and
// ringattn_protocol.h:13-60 (RingAttnBlock, RingAttnSoftmaxState, RingAttnMessage,
// RingAttnDomainConfig, RingAttnConfig). The same fields are kept so a config JSON maps 1:1;
// the message/payload structs describe the bf16 device tiles that the B200 build moves over NVLink
// instead of host byte payloads.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "hcp/core/status.h"

namespace hcp {

enum class TensorDType : int32_t { kFloat32 = 0, kFloat16 = 1, kBFloat16 = 2, kInt32 = 3, kInt64 = 4 };

inline int dtype_bytes(TensorDType t) {
  switch (t) {
    case TensorDType::kFloat32: return 4;
    case TensorDType::kFloat16: return 2;
    case TensorDType::kBFloat16: return 2;
    case TensorDType::kInt32: return 4;
    case TensorDType::kInt64: return 8;
  }
  return 0;
}

enum class TensorLayout : int32_t { kSeqHeadDim = 0, kHeadSeqDim = 1, kPaged = 2 };

// A device (or host) tensor crossing a component boundary.
struct BoundaryTensor {
  std::string name;
  TensorDType dtype = TensorDType::kBFloat16;
  TensorLayout layout = TensorLayout::kSeqHeadDim;
  std::vector<int64_t> shape;
  void* data = nullptr;   // device pointer (not owned)
  int device = -1;        // -1: host
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
  int64_t nbytes() const { return numel() * dtype_bytes(dtype); }
};

struct RingAttnBlock {
  int64_t global_offset = 0;
  int64_t block_len = 0;
  BoundaryTensor tensor;
};

struct RingAttnSoftmaxState {
  int64_t seq_len = 0;
  int64_t num_heads = 0;
  int64_t head_dim = 0;
  BoundaryTensor running_max;
  BoundaryTensor running_sum;
  BoundaryTensor output;
};

enum class RingAttnMessageType : uint32_t { kKvBlock = 1, kSoftmaxState = 2, kTerminate = 3 };

struct RingAttnMessage {
  uint64_t sequence_id = 0;
  int32_t layer_index = 0;
  int32_t source_domain_id = 0;
  int32_t target_domain_id = 0;
  RingAttnMessageType type = RingAttnMessageType::kKvBlock;
  std::vector<uint8_t> payload;
};

struct RingAttnDomainConfig {
  std::string domain_id;
  std::string host;
  int port = 0;
  int64_t seq_chunk_len = 0;
  int64_t block_size = 0;
  std::string device;
};

struct RingAttnConfig {
  int64_t global_seq_len = 0;
  int64_t num_heads = 0;
  int64_t num_kv_heads = 0;
  int64_t head_dim = 0;
  TensorDType dtype = TensorDType::kBFloat16;
  std::vector<RingAttnDomainConfig> domains;

  Status Validate() const {
    int64_t total = 0;
    for (const auto& d : domains) {
      if (d.domain_id.empty() || d.seq_chunk_len <= 0 || d.block_size <= 0)
        return Status::InvalidArgument("domain " + d.domain_id + " has invalid seq_chunk_len or block_size");
      total += d.seq_chunk_len;
    }
    if (total != global_seq_len)
      return Status::InvalidArgument("sum(seq_chunk_len)=" + std::to_string(total) +
                                     " does not match global_seq_len=" + std::to_string(global_seq_len));
    if (num_heads <= 0 || head_dim <= 0) return Status::InvalidArgument("num_heads/head_dim must be positive");
    return Status::Ok();
  }
};

}  // namespace hcp
