// Host-side per-step metadata: block-table validation and packing.
//
// Restates, in native code, what a paged step needs before its first kernel:
//   * the block-table rules of PagedAttentionMetadata.validate_block_tables
//     (runtime/execution/paged_attention.py:138-172), checked in the same
//     order with the same messages so that the first violation reported is the
//     one the reference reports;
//   * the int32 payload the kernels read, packed into one buffer for a single
//     host-to-device copy (the layout of the Triton backend's staging,
//     runtime/execution/triton_paged_attention.py:422-440): block tables padded
//     to the longest table, computed counts, query start offsets, and the
//     request index of every packed query token.
// Ownership of physical blocks across requests is tracked in thread-local
// arrays indexed by block id and stamped per call, so a call costs
// O(total blocks) without clearing anything.
#pragma once

#include <stdint.h>

#include <algorithm>
#include <vector>

namespace lvb {
namespace meta {

struct OwnerTable {
  std::vector<uint32_t> stamp;     // call id that last touched the block
  std::vector<int32_t> logical;    // logical index of its first owner
  std::vector<uint8_t> readonly;   // whether that owner marked it read-only
  std::vector<uint32_t> row_stamp; // (call, row) stamp for in-row duplicates
  uint32_t call = 0;

  void reserve(int64_t num_blocks) {
    if (static_cast<int64_t>(stamp.size()) < num_blocks) {
      stamp.assign(num_blocks, 0);
      logical.assign(num_blocks, 0);
      readonly.assign(num_blocks, 0);
      row_stamp.assign(num_blocks, 0);
      call = 0;
    }
  }
};

// Returns nullptr when valid, otherwise the reference's message.
inline const char *validate(const int32_t *block_ids, const int64_t *offsets, const int32_t *computed,
                            const int32_t *reserved, const int32_t *readonly, int64_t num_seqs,
                            int64_t num_blocks, int64_t block_size, OwnerTable &owners) {
  owners.reserve(num_blocks);
  // Stamps: one per call for ownership, one per (call, row) for duplicates.
  owners.call += 1;
  if (owners.call == 0) {  // wrapped: clear once
    std::fill(owners.stamp.begin(), owners.stamp.end(), 0u);
    std::fill(owners.row_stamp.begin(), owners.row_stamp.end(), 0u);
    owners.call = 1;
  }
  static thread_local uint32_t row_counter = 0;
  for (int64_t r = 0; r < num_seqs; ++r) {
    const int64_t begin = offsets[r];
    const int64_t len = offsets[r + 1] - begin;
    const int64_t needed = (static_cast<int64_t>(computed[r]) + reserved[r] + block_size - 1) / block_size;
    if (len < needed) return "block table does not cover all scheduled tokens";
    if (len > needed) return "block table contains unused physical blocks";
    for (int64_t i = 0; i < len; ++i)
      if (block_ids[begin + i] >= num_blocks || block_ids[begin + i] < 0)
        return "block table contains an out-of-range physical block";
    if (readonly[r] > len || static_cast<int64_t>(readonly[r]) * block_size > computed[r])
      return "readonly prefix blocks exceed the computed prefix";
    row_counter += 1;
    if (row_counter == 0) {
      std::fill(owners.row_stamp.begin(), owners.row_stamp.end(), 0u);
      row_counter = 1;
    }
    for (int64_t i = 0; i < len; ++i) {
      const int32_t b = block_ids[begin + i];
      if (owners.row_stamp[b] == row_counter) return "block table aliases a physical block within one request";
      owners.row_stamp[b] = row_counter;
    }
    for (int64_t i = 0; i < len; ++i) {
      const int32_t b = block_ids[begin + i];
      const bool ro = i < readonly[r];
      if (owners.stamp[b] == owners.call) {
        if (owners.logical[b] != i || !owners.readonly[b] || !ro)
          return "block tables alias a physical block across requests";
      }
      owners.stamp[b] = owners.call;
      owners.logical[b] = static_cast<int32_t>(i);
      owners.readonly[b] = ro ? 1 : 0;
    }
  }
  return nullptr;
}

}  // namespace meta
}  // namespace lvb
