"""CPU restatement of the reference's paged-attention path (test oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Paths in citations
are relative to the light-vllm source tree.

Cache layout (``runtime/execution/paged_cache.py:328-338``): per layer, K and
V are separate tensors shaped [num_blocks, block_size, num_kv_heads,
head_size]; a logical position p of a request lives at physical slot
``table[p // block_size] * block_size + p % block_size``.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch


class KVCacheError(RuntimeError):
    """Raised where the reference raises ``KVCacheError``
    (``runtime/kv_cache.py:21-22``)."""


def linear_parents(length: int) -> tuple[int, ...]:
    """Parent chain of an ordinary causal query block
    (``runtime/execution/layout.py:13-19``)."""

    if type(length) is not int or length <= 0:
        raise ValueError("num_queries must be a positive integer")
    return tuple(-1 if i == 0 else i - 1 for i in range(length))


def query_visibility(parents: Sequence[int]) -> tuple[tuple[bool, ...], ...]:
    """Row i marks query i itself and every ancestor on its parent chain.

    Restates ``query_visibility`` (runtime/execution/layout.py:43-55).
    """

    width = len(parents)
    rows = []
    for i, parent in enumerate(parents):
        row = [False] * width
        row[i] = True
        while parent != -1:
            row[parent] = True
            parent = parents[parent]
        rows.append(tuple(row))
    return tuple(rows)


def query_start_loc(query_lengths: Sequence[int]) -> tuple[int, ...]:
    """Prefix sums of query lengths (``paged_attention.py:77-82``)."""

    starts = [0]
    for length in query_lengths:
        starts.append(starts[-1] + length)
    return tuple(starts)


def request_indices(query_lengths: Sequence[int]) -> tuple[int, ...]:
    """Request index of every packed query token (``paged_attention.py:100-108``)."""

    return tuple(r for r, length in enumerate(query_lengths) for _ in range(length))


def slot_mapping(
    block_tables: Sequence[Sequence[int]],
    num_computed: Sequence[int],
    query_lengths: Sequence[int],
    reserved: Sequence[int],
    block_size: int,
) -> tuple[int, ...]:
    """Physical cache slot of every packed query token.

    Restates ``PagedAttentionMetadata.slot_mapping`` (paged_attention.py:110-136),
    including its coverage checks.
    """

    out: list[int] = []
    for table, computed, length, res in zip(block_tables, num_computed, query_lengths, reserved):
        needed = (computed + res + block_size - 1) // block_size
        if len(table) < needed:
            raise KVCacheError("block table does not cover all scheduled tokens")
        if len(table) > needed:
            raise KVCacheError("block table contains unused physical blocks")
        for offset in range(length):
            position = computed + offset
            out.append(table[position // block_size] * block_size + position % block_size)
    return tuple(out)


def validate_block_tables(
    block_tables: Sequence[Sequence[int]],
    num_computed: Sequence[int],
    reserved: Sequence[int],
    readonly: Sequence[int],
    *,
    num_blocks: int,
    block_size: int,
) -> None:
    """Coverage, range and aliasing rules for one step's block tables.

    Restates ``PagedAttentionMetadata.validate_block_tables``
    (paged_attention.py:138-172): exact coverage of computed + reserved
    tokens, every id below ``num_blocks``, no id twice within a request, and a
    physical block shared across requests only as the same logical index of a
    read-only prefix on both sides.
    """

    owners: dict[int, tuple[int, bool]] = {}
    for table, computed, res, n_readonly in zip(block_tables, num_computed, reserved, readonly):
        needed = (computed + res + block_size - 1) // block_size
        if len(table) < needed:
            raise KVCacheError("block table does not cover all scheduled tokens")
        if len(table) > needed:
            raise KVCacheError("block table contains unused physical blocks")
        if any(block >= num_blocks for block in table):
            raise KVCacheError("block table contains an out-of-range physical block")
        if n_readonly > len(table) or n_readonly * block_size > computed:
            raise KVCacheError("readonly prefix blocks exceed the computed prefix")
        if len(set(table)) != len(table):
            raise KVCacheError("block table aliases a physical block within one request")
        for logical, block in enumerate(table):
            is_readonly = logical < n_readonly
            prior = owners.get(block)
            if prior is not None and (prior[0] != logical or not prior[1] or not is_readonly):
                raise KVCacheError("block tables alias a physical block across requests")
            owners[block] = (logical, is_readonly)


def visibility_tensor(layouts: Sequence[Sequence[int]]) -> tuple[tuple[bool, ...], tuple[int, ...]]:
    """Flattened per-request visibility matrices and their start offsets
    (``paged_attention.py:174-186``)."""

    flat: list[bool] = []
    starts = [0]
    for parents in layouts:
        for row in query_visibility(parents):
            flat.extend(row)
        starts.append(len(flat))
    return tuple(flat), tuple(starts)


def write_slots(k_cache: torch.Tensor, v_cache: torch.Tensor, key: torch.Tensor,
                value: torch.Tensor, slots: Sequence[int]) -> None:
    """Scatter K/V rows into their slots (``paged_cache.py:208-248``)."""

    num_slots = k_cache.shape[0] * k_cache.shape[1]
    flat_k = k_cache.view(num_slots, *k_cache.shape[2:])
    flat_v = v_cache.view(num_slots, *v_cache.shape[2:])
    index = torch.tensor(list(slots), dtype=torch.long)
    flat_k.index_copy_(0, index, key)
    flat_v.index_copy_(0, index, value)


def attend(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: Sequence[Sequence[int]],
    num_computed: Sequence[int],
    layouts: Sequence[Sequence[int]],
    *,
    scale: float,
    reserved: Sequence[int] | None = None,
    write: bool = True,
) -> torch.Tensor:
    """Write this step's K/V, then attend every packed query over its pages.

    Restates ``TorchPagedAttention.forward`` / ``_attend_query_token``
    (paged_attention.py:272-380): for each query token, the visible logical
    positions are the whole computed prefix plus the query's ancestors and
    itself; they are visited page by page with an fp32 online softmax (running
    max, rescaled running sum and value), GQA by repeating each KV head over its
    query-head group, and the result is cast back to the query dtype.
    ``k_cache`` / ``v_cache`` are modified in place when ``write`` is set.
    """

    block_size = k_cache.shape[1]
    lengths = [len(p) for p in layouts]
    if reserved is None:
        reserved = lengths
    if write:
        slots = slot_mapping(block_tables, num_computed, lengths, reserved, block_size)
        write_slots(k_cache, v_cache, key, value, slots)
    num_q_heads = query.shape[1]
    num_kv_heads = k_cache.shape[2]
    repeats = num_q_heads // num_kv_heads
    acc_dtype = torch.float32 if query.dtype in (torch.float16, torch.bfloat16) else query.dtype
    out = torch.zeros_like(query)
    starts = query_start_loc(lengths)
    for row, (table, computed, parents) in enumerate(zip(block_tables, num_computed, layouts)):
        prefix = tuple(range(computed))
        for offset, visible in enumerate(query_visibility(parents)):
            positions = prefix + tuple(computed + i for i, v in enumerate(visible) if v)
            by_block: dict[int, list[int]] = {}
            for p in positions:
                by_block.setdefault(p // block_size, []).append(p % block_size)
            q = query[starts[row] + offset].to(acc_dtype)
            run_max = torch.full((num_q_heads,), -torch.inf, dtype=acc_dtype)
            run_sum = torch.zeros((num_q_heads,), dtype=acc_dtype)
            run_val = torch.zeros((num_q_heads, query.shape[2]), dtype=acc_dtype)
            for logical, offsets in by_block.items():
                block = table[logical]
                keys = k_cache[block, offsets].to(acc_dtype)
                values = v_cache[block, offsets].to(acc_dtype)
                if repeats > 1:
                    keys = keys.repeat_interleave(repeats, dim=1)
                    values = values.repeat_interleave(repeats, dim=1)
                keys = keys.permute(1, 0, 2)
                values = values.permute(1, 0, 2)
                scores = torch.einsum("hd,htd->ht", q, keys) * scale
                new_max = torch.maximum(run_max, scores.max(dim=1).values)
                rescale = torch.exp(run_max - new_max)
                weights = torch.exp(scores - new_max.unsqueeze(1))
                run_val = run_val * rescale.unsqueeze(1) + torch.einsum("ht,htd->hd", weights, values)
                run_sum = run_sum * rescale + weights.sum(dim=1)
                run_max = new_max
            out[starts[row] + offset] = (run_val / run_sum.unsqueeze(1)).to(query.dtype)
    return out


def attend_dense_fp64(
    query: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: Sequence[Sequence[int]],
    num_computed: Sequence[int],
    layouts: Sequence[Sequence[int]],
    *,
    scale: float,
) -> torch.Tensor:
    """float64 softmax attention over the same visible positions (no writes).

    A one-shot (not online) evaluation used to measure kernels at sizes where
    the page-by-page loop above is too slow; it visits exactly the positions
    ``attend`` visits.  ``k_cache``/``v_cache`` must already hold this step's
    K/V.
    """

    block_size = k_cache.shape[1]
    lengths = [len(p) for p in layouts]
    starts = query_start_loc(lengths)
    num_q_heads = query.shape[1]
    repeats = num_q_heads // k_cache.shape[2]
    out = torch.zeros(query.shape, dtype=torch.float64)
    for row, (table, computed, parents) in enumerate(zip(block_tables, num_computed, layouts)):
        table_t = torch.tensor(list(table), dtype=torch.long)
        for offset, visible in enumerate(query_visibility(parents)):
            positions = torch.tensor(
                list(range(computed)) + [computed + i for i, v in enumerate(visible) if v],
                dtype=torch.long,
            )
            blocks = table_t[positions // block_size]
            offs = positions % block_size
            keys = k_cache[blocks, offs].to(torch.float64)
            values = v_cache[blocks, offs].to(torch.float64)
            if repeats > 1:
                keys = keys.repeat_interleave(repeats, dim=1)
                values = values.repeat_interleave(repeats, dim=1)
            q = query[starts[row] + offset].to(torch.float64)
            scores = torch.einsum("hd,thd->ht", q, keys) * scale
            probs = torch.softmax(scores, dim=-1)
            out[starts[row] + offset] = torch.einsum("ht,thd->hd", probs, values)
    return out


def compact_slots(block_ids: Sequence[int], *, num_computed_tokens: int, retained_query_indices: Sequence[int],
                  block_size: int) -> tuple[tuple[int, ...], tuple[int, ...]]:
    """Source and target physical slots of ``PagedKVCache.compact``
    (runtime/execution/paged_cache.py:304-311): the retained query tokens move
    from their flattened query slots to the contiguous tail after the
    computed prefix."""

    def physical_slot(pos: int) -> int:
        return block_ids[pos // block_size] * block_size + pos % block_size

    source = tuple(physical_slot(num_computed_tokens + i) for i in retained_query_indices)
    target = tuple(physical_slot(num_computed_tokens + i) for i in range(len(retained_query_indices)))
    return source, target
