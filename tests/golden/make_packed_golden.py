"""Generates tests/golden/packed_rows.npz: a synthetic multi-shard token index and the rows that the
reference's own iterators (Midstream-LLM src/jishui/data.py:233-330 PackedBatchIterator,
:333-379 SequentialBatchIterator) produce from it. Run where the reference project is available, with
MIDSTREAM_REF naming its `src` directory (the one holding the `jishui` package):

    MIDSTREAM_REF=<reference checkout>/src python tests/golden/make_packed_golden.py
"""
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

if not os.environ.get("MIDSTREAM_REF"):
    raise SystemExit("set MIDSTREAM_REF to the reference project's src directory (it holds the jishui package)")
sys.path.insert(0, os.environ["MIDSTREAM_REF"])

from jishui.data import PackedBatchIterator, PretrainIndex, SequentialBatchIterator  # noqa: E402

OUT = Path(__file__).resolve().parent / "packed_rows.npz"


def main() -> None:
    rng = np.random.default_rng(123)
    n_docs, n_shards = 240, 3
    lengths = rng.integers(1, 900, size=n_docs).astype(np.uint32)
    shards = np.sort(rng.integers(0, n_shards, size=n_docs)).astype(np.uint8)
    offsets = np.zeros(n_docs, dtype=np.uint64)
    shard_tokens = []
    for s in range(n_shards):
        ids = np.flatnonzero(shards == s)
        pos = 0
        for i in ids:
            offsets[i] = pos
            pos += int(lengths[i])
        shard_tokens.append(rng.integers(3, 60000, size=pos).astype(np.uint16))
    categories = rng.integers(1, 7, size=n_docs).astype(np.uint8)
    categories[rng.random(n_docs) < 0.05] = 0  # unknown category: excluded from sampling
    splits = (rng.random(n_docs) < 0.2).astype(np.uint8)  # 1 = val
    sampling = {"target_mix": {str(c): float(w) for c, w in zip(range(1, 7), (0.3, 0.2, 0.15, 0.15, 0.1, 0.1))},
                "weights_by_category": {str(c): float(w) for c, w in zip(range(1, 7), (1.0, 2.0, 0.5, 1.5, 1.0, 3.0))}}
    out = {"lengths": lengths, "shards": shards, "offsets": offsets, "categories": categories, "splits": splits}
    for s, t in enumerate(shard_tokens):
        out[f"shard_{s}"] = t
    with tempfile.TemporaryDirectory() as d:
        (Path(d) / "tokens").mkdir()
        for s, t in enumerate(shard_tokens):
            np.save(Path(d) / "tokens" / f"shard_{s:05d}.npy", t)
        index = PretrainIndex(data_dir=Path(d), shards=shards, offsets=offsets, lengths=lengths,
                              categories=categories, splits=splits, sources=np.zeros(n_docs, dtype=np.uint8),
                              source_names=("synthetic",), metadata={})
        for mode in ("target", "weights"):
            it = PackedBatchIterator(index, sampling, seq_len=300, batch_size=4, seed=7, mode=mode, eod_token_id=2)
            out[f"packed_{mode}"] = np.stack([next(it) for _ in range(5)])
        seq = SequentialBatchIterator(index, "val", seq_len=300, batch_size=3, eod_token_id=2)
        out["sequential_val"] = np.stack([next(seq) for _ in range(6)])
        seq = SequentialBatchIterator(index, "val", seq_len=300, batch_size=3, eod_token_id=2, category=4)
        out["sequential_val_c4"] = np.stack([next(seq) for _ in range(6)])
    out["target_mix"] = np.asarray([sampling["target_mix"][str(c)] for c in range(1, 7)])
    out["weights_by_category"] = np.asarray([sampling["weights_by_category"][str(c)] for c in range(1, 7)])
    np.savez_compressed(OUT, **out)
    print(OUT, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
