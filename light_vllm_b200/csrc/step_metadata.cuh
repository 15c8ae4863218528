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
// Ownership of physical blocks across requests is tracked in a thread-local
// table indexed by block id and stamped per call, so a call costs
// O(total blocks) without clearing anything.
#pragma once

#include <stdint.h>

#include <algorithm>
#include <vector>

namespace lvb {
namespace meta {

// Per physical block: the (call, row) stamp of the row that last listed it
// and that row's logical index for it, shifted left once, with the row's
// read-only mark in bit 0.  Stamps grow monotonically across calls, so "listed
// earlier in this call" is "stamp >= the call's first row stamp"; one 8-byte
// record per block, read and written once per id.
struct Owner {
  uint32_t row_stamp;
  uint32_t logical_ro;
};

struct OwnerTable {
  std::vector<Owner> blocks;
  uint32_t row = 0;  // last (call, row) stamp handed out

  void reserve(int64_t num_blocks) {
    if (static_cast<int64_t>(blocks.size()) < num_blocks) {
      blocks.assign(num_blocks, Owner{0, 0});
      row = 0;
    }
  }
};

// The rules of one row in the reference's order, without the fast path's
// shortcuts; called only once the fused pass has seen a violation in row r
// (rows before r passed, so their stamps are intact).  Row r's own records
// may be partly rewritten, which only the in-row duplicate rule could notice,
// and that rule uses a fresh stamp here.
inline const char *row_violation(const int32_t *ids, int64_t len, int64_t needed, int32_t computed,
                                 int32_t readonly, int64_t num_blocks, int64_t block_size, OwnerTable &owners,
                                 uint32_t row_stamp) {
  if (len < needed) return "block table does not cover all scheduled tokens";
  if (len > needed) return "block table contains unused physical blocks";
  for (int64_t i = 0; i < len; ++i)
    if (ids[i] >= num_blocks || ids[i] < 0) return "block table contains an out-of-range physical block";
  if (readonly > len || static_cast<int64_t>(readonly) * block_size > computed)
    return "readonly prefix blocks exceed the computed prefix";
  Owner *own = owners.blocks.data();
  for (int64_t i = 0; i < len; ++i) {
    if (own[ids[i]].row_stamp == row_stamp) return "block table aliases a physical block within one request";
    own[ids[i]].row_stamp = row_stamp;
  }
  return "block tables alias a physical block across requests";
}

// Returns nullptr when valid, otherwise the reference's message.  Valid rows
// take one fused pass per id (range, in-row duplicate, cross-row ownership);
// the first violation sends its row through row_violation, which applies the
// rules in the reference's order and so reports the same message.  A block
// may appear in several rows only inside their read-only prefixes, at the
// same logical index.
inline const char *validate(const int32_t *block_ids, const int64_t *offsets, const int32_t *computed,
                            const int32_t *reserved, const int32_t *readonly, int64_t num_seqs,
                            int64_t num_blocks, int64_t block_size, OwnerTable &owners) {
  owners.reserve(num_blocks);
  // Stamps are uint32: a call needs num_seqs + 2 of them; wrap-around clears
  // the table once.
  if (owners.row > UINT32_MAX - static_cast<uint32_t>(num_seqs) - 2) {
    std::fill(owners.blocks.begin(), owners.blocks.end(), Owner{0, 0});
    owners.row = 0;
  }
  uint32_t row = owners.row;
  const uint32_t first = row + 1;  // stamps >= first were handed out in this call
  Owner *own = owners.blocks.data();
  const char *violation = nullptr;
  for (int64_t r = 0; r < num_seqs && violation == nullptr; ++r) {
    const int32_t *ids = block_ids + offsets[r];
    const int64_t len = offsets[r + 1] - offsets[r];
    const int64_t needed = (static_cast<int64_t>(computed[r]) + reserved[r] + block_size - 1) / block_size;
    const int32_t ro_len = readonly[r];
    const uint32_t rs = ++row;
    bool ok = len == needed && ro_len <= len && static_cast<int64_t>(ro_len) * block_size <= computed[r];
    for (int64_t i = 0; ok && i < len; ++i) {
      const int32_t b = ids[i];
      if (b < 0 || b >= num_blocks) {
        ok = false;
        break;
      }
      const Owner o = own[b];
      const uint32_t mine = (static_cast<uint32_t>(i) << 1) | (i < ro_len ? 1u : 0u);
      // Listed before in this call: a duplicate in this row, or another row's
      // block that may be shared only as the same read-only prefix block.
      if (o.row_stamp >= first && (o.row_stamp == rs || (mine & 1u) == 0u || o.logical_ro != mine)) {
        ok = false;
        break;
      }
      own[b] = Owner{rs, mine};
    }
    if (!ok) violation = row_violation(ids, len, needed, computed[r], ro_len, num_blocks, block_size, owners, ++row);
  }
  owners.row = row;
  return violation;
}

}  // namespace meta
}  // namespace lvb
