"""Stand-ins for light-vllm's paged-KV interface types (test infrastructure).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  The B200 backend
plugs in behind ``PagedAttentionBackend.create(cache, metadata)``
(runtime/execution/paged_attention.py:216-223) and touches the cache and the
metadata only through the attributes and methods the reference defines, so it
takes the reference's own ``PagedKVCache`` and ``PagedAttentionMetadata``.
The tests, ``smoke()`` and the bench use those when light-vllm is importable
(``reference_types()``); where it is not (the GPU box ships without it unless
``baseline/_ref`` travelled), this module restates the same types with the
same names, fields, rules and messages:

  AttentionLayerSpec, ModelKVCacheSpec   modeling/attention/interfaces.py:9-45
  QueryLayout                            runtime/execution/interfaces.py:82-97
  linear_query_layout, query_visibility  runtime/execution/layout.py:13-55
  KVCacheCapacityError                   runtime/kv_cache.py:21-26
  PagedKVCacheConfig, PagedKVCache,      runtime/execution/paged_cache.py:30-338
    kv_cache_bytes_per_block
  PagedAttentionMetadata                 runtime/execution/paged_attention.py:18-206

Cache writes are the reference's ``index_copy_``; nothing here calls the
sm_100a library.
"""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass
from pathlib import Path
from types import SimpleNamespace

import torch
from torch import Tensor

from oracle.paged_attention import KVCacheError

_ROOT = Path(__file__).resolve().parents[1]


def reference_types() -> SimpleNamespace:
    """The reference's own paged-KV classes when light-vllm is importable --
    from ``LIGHT_VLLM_SRC`` or the offline install under ``baseline/_ref`` --
    else this module's stand-ins.  ``.source`` says which."""

    for candidate in (os.environ.get("LIGHT_VLLM_SRC"), str(_ROOT / "baseline" / "_ref")):
        if candidate and Path(candidate, "light_vllm").is_dir() and candidate not in sys.path:
            sys.path.append(candidate)
    try:
        from light_vllm.modeling.attention import AttentionLayerSpec as RSpec
        from light_vllm.modeling.attention import ModelKVCacheSpec as RModel
        from light_vllm.runtime.execution.interfaces import QueryLayout as RLayout
        from light_vllm.runtime.execution.layout import linear_query_layout as rlinear
        from light_vllm.runtime.execution.paged_attention import PagedAttentionMetadata as RMeta
        from light_vllm.runtime.execution.paged_cache import PagedKVCache as RCache
        from light_vllm.runtime.execution.paged_cache import PagedKVCacheConfig as RConfig
        from light_vllm.runtime.kv_cache import KVCacheError as RError
    except ImportError:
        return SimpleNamespace(source="oracle", AttentionLayerSpec=AttentionLayerSpec,
                               ModelKVCacheSpec=ModelKVCacheSpec, QueryLayout=QueryLayout,
                               linear_query_layout=linear_query_layout, PagedAttentionMetadata=PagedAttentionMetadata,
                               PagedKVCache=PagedKVCache, PagedKVCacheConfig=PagedKVCacheConfig,
                               KVCacheError=KVCacheError)
    return SimpleNamespace(source="light_vllm", AttentionLayerSpec=RSpec, ModelKVCacheSpec=RModel,
                           QueryLayout=RLayout, linear_query_layout=rlinear, PagedAttentionMetadata=RMeta,
                           PagedKVCache=RCache, PagedKVCacheConfig=RConfig, KVCacheError=RError)


def model_spec(types: SimpleNamespace, layers) -> object:
    """``ModelKVCacheSpec`` of ``types`` over (layer_id, query heads, KV heads,
    head size) tuples (``Qwen2AWQRunner.kv_layers()``)."""

    return types.ModelKVCacheSpec(tuple(types.AttentionLayerSpec(*layer) for layer in layers))


class KVCacheCapacityError(KVCacheError):
    """Not enough KV slots for the requested reservation."""


@dataclass(frozen=True, slots=True)
class AttentionLayerSpec:
    """Logical K/V shape of one attention layer."""

    layer_id: str
    num_query_heads: int
    num_kv_heads: int
    head_size: int

    def __post_init__(self) -> None:
        if not self.layer_id:
            raise ValueError("layer_id must not be empty")
        for name in ("num_query_heads", "num_kv_heads", "head_size"):
            value = getattr(self, name)
            if type(value) is not int or value <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if self.num_query_heads % self.num_kv_heads != 0:
            raise ValueError("num_query_heads must be divisible by num_kv_heads")


@dataclass(frozen=True, slots=True)
class ModelKVCacheSpec:
    """K/V shapes of every cacheable attention layer of a model."""

    layers: tuple[AttentionLayerSpec, ...]

    def __post_init__(self) -> None:
        layers = tuple(self.layers)
        if not layers:
            raise ValueError("model KV cache spec must contain at least one layer")
        ids = [layer.layer_id for layer in layers]
        if len(set(ids)) != len(ids):
            raise ValueError("attention layer IDs must be unique")
        object.__setattr__(self, "layers", layers)


@dataclass(frozen=True, slots=True)
class QueryLayout:
    """Parent of each query of one step (-1 = attaches to the committed prefix)."""

    parent_indices: tuple[int, ...]

    def __post_init__(self) -> None:
        parents = tuple(self.parent_indices)
        if not parents:
            raise ValueError("query layout must not be empty")
        for index, parent in enumerate(parents):
            if type(parent) is not int or not -1 <= parent < index:
                raise ValueError("each query parent must be -1 or precede its child")
        object.__setattr__(self, "parent_indices", parents)

    def __len__(self) -> int:
        return len(self.parent_indices)


def linear_query_layout(num_queries: int) -> QueryLayout:
    """The ordinary causal chain of ``num_queries`` queries."""

    if type(num_queries) is not int or num_queries <= 0:
        raise ValueError("num_queries must be a positive integer")
    return QueryLayout(tuple(range(-1, num_queries - 1)))


def query_visibility(layout: QueryLayout) -> tuple[tuple[bool, ...], ...]:
    """Row i is true at query i and at each ancestor of query i."""

    parents = layout.parent_indices
    width = len(parents)
    rows = []
    for index in range(width):
        row = [False] * width
        node = index
        while node != -1:
            row[node] = True
            node = parents[node]
        rows.append(tuple(row))
    return tuple(rows)


@dataclass(frozen=True, slots=True)
class PagedKVCacheConfig:
    """A decided paged-cache configuration (also usable as its own planner)."""

    num_blocks: int
    block_size: int
    dtype: torch.dtype = torch.float32
    device: str | torch.device = "cpu"

    def __post_init__(self) -> None:
        if type(self.num_blocks) is not int or self.num_blocks <= 0:
            raise ValueError("num_blocks must be a positive integer")
        if type(self.block_size) is not int or self.block_size <= 0:
            raise ValueError("block_size must be a positive integer")
        if not self.dtype.is_floating_point:
            raise ValueError("KV cache dtype must be floating point")
        object.__setattr__(self, "device", torch.device(self.device))

    def plan(self, model_spec: ModelKVCacheSpec) -> "PagedKVCacheConfig":
        return self


def kv_cache_bytes_per_block(model_spec: ModelKVCacheSpec, *, block_size: int,
                             dtype: torch.dtype) -> int:
    """Bytes of one physical block across all layers (K and V)."""

    per_token = sum(2 * layer.num_kv_heads * layer.head_size for layer in model_spec.layers)
    return block_size * per_token * torch.empty((), dtype=dtype).element_size()


@dataclass(frozen=True, slots=True)
class PagedLayerCache:
    """One layer's K and V, each [num_blocks, block_size, num_kv_heads, head_size]."""

    keys: Tensor
    values: Tensor


@dataclass(frozen=True, slots=True)
class PagedKVWriteMapping:
    """Physical slots of one step's packed query tokens, reused by every layer."""

    slots: Tensor
    num_query_tokens: int
    source_indices: Tensor | None = None


class PagedKVCache:
    """Per-layer paged K/V pools addressed by shared physical block ids."""

    def __init__(self, model_spec: ModelKVCacheSpec, config: PagedKVCacheConfig) -> None:
        self._model_spec = model_spec
        self._config = config
        self._layer_specs = {layer.layer_id: layer for layer in model_spec.layers}
        self._layers = {layer.layer_id: self._allocate_layer(layer) for layer in model_spec.layers}

    @property
    def config(self) -> PagedKVCacheConfig:
        return self._config

    @property
    def model_spec(self) -> ModelKVCacheSpec:
        return self._model_spec

    def layer_spec(self, layer_id: str) -> AttentionLayerSpec:
        try:
            return self._layer_specs[layer_id]
        except KeyError as exc:
            raise KVCacheError(f"KV cache layer {layer_id!r} was not found") from exc

    def layer(self, layer_id: str) -> PagedLayerCache:
        try:
            return self._layers[layer_id]
        except KeyError as exc:
            raise KVCacheError(f"KV cache layer {layer_id!r} was not found") from exc

    def prepare_write(self, slot_mapping: Tensor, *, validate: bool = True) -> PagedKVWriteMapping:
        """Normalise a slot mapping once per step (negative slots are skipped)."""

        if slot_mapping.ndim != 1:
            raise KVCacheError("slot mapping must have one entry per packed query token")
        if slot_mapping.device != self._config.device:
            raise KVCacheError("slot mapping device must match the cache")
        if not validate:
            return PagedKVWriteMapping(slot_mapping.to(torch.long), slot_mapping.numel())
        active = slot_mapping >= 0
        source = torch.nonzero(active, as_tuple=False).flatten()
        slots = slot_mapping.index_select(0, source).to(torch.long)
        if slots.numel():
            num_slots = self._config.num_blocks * self._config.block_size
            if int(slots.min()) < 0 or int(slots.max()) >= num_slots:
                raise KVCacheError("slot mapping contains an out-of-range physical slot")
            if slots.unique().numel() != slots.numel():
                raise KVCacheError("slot mapping must not write the same physical slot twice")
        return PagedKVWriteMapping(
            slots,
            slot_mapping.numel(),
            None if source.numel() == slot_mapping.numel() else source,
        )

    def write_prepared(self, layer_id: str, key: Tensor, value: Tensor,
                       mapping: PagedKVWriteMapping) -> None:
        """Copy K/V rows into the prepared slots (``index_copy_`` on a flat
        [slots, heads, dim] view, as the reference does)."""

        layer = self.layer(layer_id)
        spec = self.layer_spec(layer_id)
        tail = (spec.num_kv_heads, spec.head_size)
        if key.ndim != 3 or tuple(key.shape[1:]) != tail:
            raise KVCacheError("paged KV update must have shape [tokens, kv_heads, head_size]")
        if value.shape != key.shape:
            raise KVCacheError("paged K/V updates must have the same shape")
        if mapping.num_query_tokens != key.shape[0]:
            raise KVCacheError("slot mapping must have one entry per query token")
        if key.dtype != self._config.dtype or key.device != self._config.device:
            raise KVCacheError("paged KV update dtype and device must match the cache")
        if value.dtype != key.dtype or value.device != key.device:
            raise KVCacheError("paged K/V updates must use the same dtype and device")
        if mapping.slots.numel() == 0:
            return
        if mapping.source_indices is not None:
            key = key.index_select(0, mapping.source_indices)
            value = value.index_select(0, mapping.source_indices)
        num_slots = self._config.num_blocks * self._config.block_size
        layer.keys.view(num_slots, *tail).index_copy_(0, mapping.slots, key)
        layer.values.view(num_slots, *tail).index_copy_(0, mapping.slots, value)

    def write(self, layer_id: str, key: Tensor, value: Tensor, slot_mapping: Tensor) -> None:
        """Write valid query tokens' K/V to the given physical slots."""

        self.write_prepared(layer_id, key, value, self.prepare_write(slot_mapping))

    def compact(self, block_ids: tuple[int, ...], *, num_computed_tokens: int, num_query_tokens: int,
                num_reserved_query_tokens: int, retained_query_indices: tuple[int, ...],
                num_readonly_prefix_blocks: int = 0) -> int:
        """Move the retained query tokens' K/V from their flattened query slots
        to the contiguous tail after the computed prefix; returns how many
        tokens moved (runtime/execution/paged_cache.py:257-326)."""

        block_ids = tuple(block_ids)
        retained = tuple(retained_query_indices)
        values = (num_computed_tokens, num_query_tokens, num_reserved_query_tokens, num_readonly_prefix_blocks)
        if any(type(v) is not int or v < 0 for v in values):
            raise ValueError("paged compact counts must be non-negative integers")
        if num_reserved_query_tokens < num_query_tokens:
            raise ValueError("reserved query tokens must cover every actual query")
        if any(type(i) is not int or i < 0 for i in retained):
            raise ValueError("retained query indices must be non-negative integers")
        if len(set(retained)) != len(retained):
            raise ValueError("retained query indices must be unique")
        if any(i >= num_query_tokens for i in retained):
            raise KVCacheError("retained query index exceeds the paged KV tail")
        config = self._config
        required = (num_computed_tokens + num_reserved_query_tokens + config.block_size - 1) // config.block_size
        if len(block_ids) != required:
            raise KVCacheError("block table does not exactly cover the reserved query slots")
        if any(type(b) is not int or not 0 <= b < config.num_blocks for b in block_ids):
            raise KVCacheError("block table contains an invalid physical block")
        if len(set(block_ids)) != len(block_ids):
            raise KVCacheError("block table aliases a physical block within one request")
        if num_readonly_prefix_blocks * config.block_size > num_computed_tokens:
            raise KVCacheError("readonly prefix blocks exceed the computed prefix")

        def physical_slot(pos: int) -> int:
            return block_ids[pos // config.block_size] * config.block_size + pos % config.block_size

        source_slots = tuple(physical_slot(num_computed_tokens + i) for i in retained)
        target_slots = tuple(physical_slot(num_computed_tokens + i) for i in range(len(retained)))
        if source_slots == target_slots:
            return 0
        source = torch.tensor(source_slots, dtype=torch.long, device=config.device)
        target = torch.tensor(target_slots, dtype=torch.long, device=config.device)
        num_slots = config.num_blocks * config.block_size
        for layer in self._layers.values():
            flat_keys = layer.keys.view(num_slots, *layer.keys.shape[2:])
            flat_values = layer.values.view(num_slots, *layer.values.shape[2:])
            keys = flat_keys.index_select(0, source).clone()  # every source read before any target is written
            values_ = flat_values.index_select(0, source).clone()
            flat_keys.index_copy_(0, target, keys)
            flat_values.index_copy_(0, target, values_)
        return sum(a != b for a, b in zip(source_slots, target_slots))

    def _allocate_layer(self, spec: AttentionLayerSpec) -> PagedLayerCache:
        shape = (self._config.num_blocks, self._config.block_size, spec.num_kv_heads, spec.head_size)
        return PagedLayerCache(
            keys=torch.empty(shape, dtype=self._config.dtype, device=self._config.device),
            values=torch.empty(shape, dtype=self._config.dtype, device=self._config.device),
        )


@dataclass(frozen=True, slots=True)
class PagedAttentionMetadata:
    """Facts one packed query batch needs to read and write paged K/V."""

    block_tables: tuple[tuple[int, ...], ...]
    num_computed_tokens: tuple[int, ...]
    query_layouts: tuple[QueryLayout, ...]
    num_reserved_query_tokens: tuple[int, ...] = ()
    num_readonly_prefix_blocks: tuple[int, ...] = ()

    def __post_init__(self) -> None:
        tables = tuple(tuple(table) for table in self.block_tables)
        computed = tuple(self.num_computed_tokens)
        layouts = tuple(self.query_layouts)
        reserved = tuple(self.num_reserved_query_tokens)
        readonly = tuple(self.num_readonly_prefix_blocks)
        n = len(tables)
        if n == 0:
            raise ValueError("paged attention metadata must contain at least one request")
        if len(computed) != n or len(layouts) != n:
            raise ValueError("paged attention metadata fields must have the same batch size")
        if not reserved:
            reserved = tuple(len(layout) for layout in layouts)
        if len(reserved) != n:
            raise ValueError("reserved query counts must have the same batch size")
        if not readonly:
            readonly = (0,) * n
        if len(readonly) != n:
            raise ValueError("readonly prefix counts must have the same batch size")
        if any(type(v) is not int or v < 0 for v in computed):
            raise ValueError("computed-token counts must be non-negative integers")
        if any(type(v) is not int or v < len(layout) for v, layout in zip(reserved, layouts)):
            raise ValueError("reserved query counts must cover every actual query")
        if any(type(v) is not int or v < 0 for v in readonly):
            raise ValueError("readonly prefix counts must be non-negative integers")
        if any(type(b) is not int or b < 0 for table in tables for b in table):
            raise ValueError("block tables must contain non-negative integers")
        object.__setattr__(self, "block_tables", tables)
        object.__setattr__(self, "num_computed_tokens", computed)
        object.__setattr__(self, "query_layouts", layouts)
        object.__setattr__(self, "num_reserved_query_tokens", reserved)
        object.__setattr__(self, "num_readonly_prefix_blocks", readonly)

    @property
    def batch_size(self) -> int:
        return len(self.block_tables)

    @property
    def query_lengths(self) -> tuple[int, ...]:
        return tuple(len(layout) for layout in self.query_layouts)

    @property
    def query_start_loc(self) -> tuple[int, ...]:
        starts = [0]
        for length in self.query_lengths:
            starts.append(starts[-1] + length)
        return tuple(starts)

    @property
    def num_query_tokens(self) -> int:
        return sum(self.query_lengths)

    @property
    def has_only_linear_queries(self) -> bool:
        return all(
            layout.parent_indices == tuple(range(-1, len(layout) - 1))
            for layout in self.query_layouts
        )

    @property
    def request_indices(self) -> tuple[int, ...]:
        out: list[int] = []
        for request, length in enumerate(self.query_lengths):
            out.extend([request] * length)
        return tuple(out)

    def _required_blocks(self, row: int, block_size: int) -> int:
        total = self.num_computed_tokens[row] + self.num_reserved_query_tokens[row]
        return -(-total // block_size)

    def _check_coverage(self, row: int, block_size: int) -> None:
        needed = self._required_blocks(row, block_size)
        have = len(self.block_tables[row])
        if have < needed:
            raise KVCacheError("block table does not cover all scheduled tokens")
        if have > needed:
            raise KVCacheError("block table contains unused physical blocks")

    def slot_mapping(self, *, block_size: int, device: torch.device) -> Tensor:
        """Physical slot of every packed query token."""

        slots: list[int] = []
        for row, (table, computed, layout) in enumerate(
            zip(self.block_tables, self.num_computed_tokens, self.query_layouts)
        ):
            self._check_coverage(row, block_size)
            for position in range(computed, computed + len(layout)):
                slots.append(table[position // block_size] * block_size + position % block_size)
        return torch.tensor(slots, dtype=torch.long, device=device)

    def validate_block_tables(self, *, num_blocks: int, block_size: int) -> None:
        """Coverage, range and aliasing rules for every table of the step."""

        owners: dict[int, tuple[int, bool]] = {}
        for row, (table, computed, n_readonly) in enumerate(
            zip(self.block_tables, self.num_computed_tokens, self.num_readonly_prefix_blocks)
        ):
            self._check_coverage(row, block_size)
            if any(block >= num_blocks for block in table):
                raise KVCacheError("block table contains an out-of-range physical block")
            if n_readonly > len(table) or n_readonly * block_size > computed:
                raise KVCacheError("readonly prefix blocks exceed the computed prefix")
            if len(set(table)) != len(table):
                raise KVCacheError("block table aliases a physical block within one request")
            for logical, block in enumerate(table):
                shared = logical < n_readonly
                seen = owners.get(block)
                if seen is not None and (seen[0] != logical or not seen[1] or not shared):
                    raise KVCacheError("block tables alias a physical block across requests")
                owners[block] = (logical, shared)

    def visibility_tensor(self, *, device: torch.device) -> tuple[Tensor, Tensor]:
        """Packed per-request visibility matrices and their start offsets."""

        flat: list[bool] = []
        starts = [0]
        for layout in self.query_layouts:
            for row in query_visibility(layout):
                flat.extend(row)
            starts.append(len(flat))
        return (
            torch.tensor(flat, dtype=torch.bool, device=device),
            torch.tensor(starts, dtype=torch.int32, device=device),
        )

    def request_indices_tensor(self, *, device: torch.device) -> Tensor:
        return torch.tensor(self.request_indices, dtype=torch.int32, device=device)

    def visible_logical_positions(self, row: int) -> tuple[tuple[int, ...], ...]:
        """Logical positions each query of request ``row`` may read."""

        computed = self.num_computed_tokens[row]
        prefix = tuple(range(computed))
        return tuple(
            prefix + tuple(computed + i for i, seen in enumerate(visible) if seen)
            for visible in query_visibility(self.query_layouts[row])
        )
