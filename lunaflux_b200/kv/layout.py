"""KV cache layout planner.

Reference: kv/device_layout/planner.mbt:69-128 (canonical V1 layout
``[layer][K/V][page][token][kv_head][head_dim]``, checked strides).  This
framework uses layout version 2, ``[layer][K/V][page][kv_head][token][dim]``:
one (page, kv head) block of 16 x 128 bf16 is 4 KB contiguous, so the
attention kernels fetch it with one TMA box pair.  The layout version is part
of the prefix-cache identity.
"""
from __future__ import annotations

import dataclasses

from ..models.spec import LlamaSpec

LAYOUT_VERSION = 2


@dataclasses.dataclass(frozen=True)
class KVLayout:
    layers: int
    kv_heads: int
    tokens_per_page: int
    head_dim: int
    elem_bytes: int = 2

    @property
    def page_component_bytes(self) -> int:
        """Bytes of one (layer, K or V, page) slab."""
        return self.kv_heads * self.tokens_per_page * self.head_dim * self.elem_bytes

    @property
    def bytes_per_page(self) -> int:
        """Bytes of one page across all layers, K and V."""
        return self.layers * 2 * self.page_component_bytes

    def element_offset(self, num_pages: int, layer: int, kv: int, page: int, head: int, token: int, dim: int) -> int:
        for v, n in ((kv, 2), (head, self.kv_heads), (token, self.tokens_per_page), (dim, self.head_dim),
                     (layer, self.layers), (page, num_pages)):
            if not (0 <= v < n):
                raise IndexError("KV coordinate out of range")
        return ((((layer * 2 + kv) * num_pages + page) * self.kv_heads + head) * self.tokens_per_page
                + token) * self.head_dim + dim


def kv_bytes_per_page(spec: LlamaSpec, kv_heads_local: int, tokens_per_page: int = 16, elem_bytes: int = 2) -> int:
    return KVLayout(spec.layers, kv_heads_local, tokens_per_page, spec.head_dim, elem_bytes).bytes_per_page
