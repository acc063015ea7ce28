"""lorafusion_b200: lorafusion's fused multi-adapter LoRA operator, rebuilt for NVIDIA B200 (sm_100a).

* :mod:`lorafusion_b200.b200_ops` — ``fused_lora_forward`` / ``fused_lora_backward``,
  the drop-in backend (same API as ``lorafusion.ops.mock_ops``).
* :mod:`lorafusion_b200.config` — ``AdapterSpec``, ``TileRoute``, ``TileRoutingConfig``.
* :mod:`lorafusion_b200.scheduler` — grouping, bin packing and fused-batch assembly.
* :mod:`lorafusion_b200.coordinator` — ``Coordinator`` (request batch in, results out).
* :mod:`lorafusion_b200.sharding` — row sharding of packed bins across GPUs and the
  gradient all-reduce of adapters that span ranks.
"""

__version__ = "0.1.0"

from lorafusion_b200.config import AdapterSpec, TileRoute, TileRoutingConfig  # noqa: F401
