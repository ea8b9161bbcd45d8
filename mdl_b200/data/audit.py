"""Feature cardinality audit (reference ``FeatureCardinalityAuditor`` /
``run_feature_cardinality_audit``, ``src/dataloader.py:4679-4740, 7468``).

Samples up to ``max_rows`` raw rows of a split and, for every categorical
feature, measures how many values each row carries: a feature configured as a
single value (``pooling: none``) whose column holds lists with more than one
element is reported as a *scalar multi* (its extra values would be dropped);
bags report their length distribution. Lengths come from the Arrow list
offsets, column by column, without converting rows to Python objects.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class FieldStats:
    rows: int = 0
    nulls: int = 0
    multi: int = 0          # rows with more than one value
    max_len: int = 0
    total_len: int = 0
    samples: list = field(default_factory=list)

    def payload(self) -> dict:
        return {"rows": self.rows, "nulls": self.nulls, "multi_rows": self.multi, "max_len": self.max_len,
                "mean_len": round(self.total_len / max(1, self.rows - self.nulls), 4), "samples": self.samples}


def _lengths(col) -> tuple[np.ndarray, np.ndarray, object]:
    """Per-row value counts, a null mask and the flat values of one Arrow column."""

    import pyarrow as pa
    import pyarrow.compute as pc

    col = col.combine_chunks() if isinstance(col, pa.ChunkedArray) else col
    nulls = np.asarray(col.is_null().to_numpy(zero_copy_only=False), dtype=bool)
    if pa.types.is_list(col.type) or pa.types.is_large_list(col.type):
        lens = np.asarray(pc.fill_null(pc.list_value_length(col), 0).to_numpy(zero_copy_only=False))
        return lens, nulls, col
    return np.where(nulls, 0, 1), nulls, None


def audit_cardinality(config, paths, max_rows: int = 100_000, samples: int = 3) -> dict:
    import pyarrow.parquet as pq

    cats = [f for f in config.features if f.kind == "categorical"]
    scalar = {f.source or f.name: f.name for f in cats if f.pooling == "none"}
    bags = {f.source or f.name: f.name for f in cats if f.pooling != "none"}
    stats: dict[str, FieldStats] = {}
    seen = 0
    for path in paths:
        if seen >= max_rows:
            break
        pf = pq.ParquetFile(path)
        cols = [c for c in {**scalar, **bags} if c in pf.schema_arrow.names]
        for g in range(pf.metadata.num_row_groups):
            if seen >= max_rows:
                break
            table = pf.read_row_group(g, columns=cols).slice(0, max_rows - seen)
            seen += table.num_rows
            for c in cols:
                lens, nulls, lst = _lengths(table.column(c))
                st = stats.setdefault(c, FieldStats())
                st.rows += len(lens)
                st.nulls += int(nulls.sum())
                st.total_len += int(lens.sum())
                st.max_len = max(st.max_len, int(lens.max()) if len(lens) else 0)
                multi = np.nonzero(lens > 1)[0]
                st.multi += len(multi)
                if c in scalar and lst is not None:
                    for i in multi[:max(0, samples - len(st.samples))]:
                        st.samples.append(lst[int(i)].as_py()[:8])
    scalar_multis = sorted(scalar[c] for c, st in stats.items() if c in scalar and st.multi)
    return {"raw_rows_seen": seen,
            "scalar_stats": {scalar[c]: st.payload() for c, st in sorted(stats.items()) if c in scalar},
            "bag_stats": {bags[c]: st.payload() for c, st in sorted(stats.items()) if c in bags},
            "scalar_multis": scalar_multis, "passed": not scalar_multis}
