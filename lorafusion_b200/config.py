"""Routing contract shared by the scheduler and the fused multi-adapter LoRA op.

Same public names, fields and error behaviour as lorafusion's
``lorafusion/ops/config.py`` (AdapterSpec ``:14-26``, TileRoute ``:29-39``,
TileRoutingConfig ``:42-69``), so objects built by either package can be
passed to either package's op.  The op in :mod:`lorafusion_b200.b200_ops`
only relies on the duck-typed attributes (``routes``, ``row_start``,
``row_end``, ``adapter_id``, ``scaling``, ``validate``), which means the
reference's own dataclasses work unchanged as inputs.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class AdapterSpec:
    """One LoRA adapter: its rank, its alpha and the projection it patches.

    ``scaling`` is ``alpha / rank`` (lorafusion/ops/config.py:24-26).
    """

    adapter_id: int
    rank: int
    alpha: float
    in_features: int
    out_features: int

    @property
    def scaling(self) -> float:
        return self.alpha / self.rank


@dataclass(frozen=True)
class TileRoute:
    """A half-open range ``[row_start, row_end)`` of fused rows owned by one adapter."""

    row_start: int
    row_end: int
    adapter_id: int

    @property
    def num_rows(self) -> int:
        return self.row_end - self.row_start


@dataclass(frozen=True)
class TileRoutingConfig:
    """The routing plan of one fused batch: ordered, contiguous adapter row ranges.

    ``tile_size`` is the packer's bin capacity.  ``num_tiles`` counts
    ``ceil(rows / tile_size)`` per route, which is not the bin count
    (lorafusion/ops/config.py:49-53).
    """

    tile_size: int
    routes: list[TileRoute] = field(default_factory=list)

    def num_tiles(self) -> int:
        ts = self.tile_size
        return sum(-(-r.num_rows // ts) for r in self.routes)

    def validate(self, total_rows: int) -> None:
        """Raise ``ValueError`` unless the routes tile ``[0, total_rows)`` in order.

        Mirrors lorafusion/ops/config.py:55-69: the first route whose start is
        not the previous end reports a gap/overlap; otherwise a mismatch in
        covered rows reports under- or over-coverage.
        """
        expected_start = 0
        covered = 0
        for r in self.routes:
            if r.row_start != expected_start:
                raise ValueError(
                    f"Routing gap/overlap at row {r.row_start}, expected {expected_start}"
                )
            covered += r.row_end - r.row_start
            expected_start = r.row_end
        if covered != total_rows:
            raise ValueError(f"Routing covers {covered} rows, expected {total_rows}")
