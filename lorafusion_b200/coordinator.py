"""Request-batch-in, per-request-results-out runtime over the fused op.

Same constructor and ``run_batch`` contract as lorafusion's
``lorafusion/runtime/coordinator.py:21-67``: bucket requests by adapter, pack
per-adapter row counts into tiles (greedy, or exact when asked and PuLP is
available), assemble the fused batch, run ``backend.fused_lora_forward`` and
scatter the fused rows back per request.  The default backend is this
package's B200 op; any module with the same two functions (the reference's
``mock_ops``/``triton_ops`` included) can be passed instead.
"""

from __future__ import annotations

from types import ModuleType

import torch

from lorafusion_b200 import b200_ops
from lorafusion_b200.config import AdapterSpec
from lorafusion_b200.scheduler import Request, build_microbatch, bucket_by_adapter, greedy_pack, milp_pack, \
    scatter_outputs


class Coordinator:
    """Serves a list of requests, each tied to one adapter, with a single call of the backend's
    fused forward: the requests' rows are packed into tiles, the op runs once on the packed batch,
    and each request gets its own rows of the result back (keyed by request id)."""

    def __init__(
        self,
        base_weight: torch.Tensor,
        adapters: dict[int, AdapterSpec],
        lora_a: dict[int, torch.Tensor],
        lora_b: dict[int, torch.Tensor],
        tile_capacity: int = 128,
        use_milp: bool = False,
        backend: ModuleType = b200_ops,
    ) -> None:
        self.base_weight = base_weight
        self.adapters = adapters
        self.lora_a = lora_a
        self.lora_b = lora_b
        self.tile_capacity = tile_capacity
        self.use_milp = use_milp
        self.backend = backend

    def run_batch(
        self, requests: list[Request], request_tensors: dict[int, torch.Tensor]
    ) -> dict[int, torch.Tensor]:
        rows = {g.adapter_id: g.total_rows for g in bucket_by_adapter(requests)}
        packing = (milp_pack if self.use_milp else greedy_pack)(rows, self.tile_capacity)
        fused_x, routing, row_order = build_microbatch(requests, request_tensors, packing)
        fused_out = self.backend.fused_lora_forward(
            fused_x, self.base_weight, self.lora_a, self.lora_b, self.adapters, routing)
        return scatter_outputs(fused_out, row_order)
