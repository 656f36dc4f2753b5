"""Writes tests/golden/known_answers.json.

Every case is a known-answer test transcribed (as data) from VectorAccelerate's own XCTest
suite; ``source`` gives the test file and line range inside the reference project. Inputs and
expected outputs are exactly the values those tests assert. The reference cannot run here (Swift
+ Metal on macOS), so these transcribed expectations are the pins for the CPU oracle
(tests/test_oracle_golden.py) and the CUDA library (tests/test_gpu_parity.py).

Run: python tests/golden/make_golden.py
"""

import json
import os

CASES = [
    # ---------------------------------------------------------------- flat L2^2 search
    {"kind": "knn", "metric": "l2", "source": "Tests/VectorAccelerateTests/KernelTests.swift:806-835",
     "queries": [[0, 0, 0, 0]],
     "database": [[1, 0, 0, 0], [2, 0, 0, 0], [0.5, 0, 0, 0], [3, 0, 0, 0]],
     "k": 2, "ids": [[2, 0]], "values": [[0.25, 1.0]], "tol": 1e-4},
    {"kind": "knn", "metric": "l2", "source": "Tests/VectorAccelerateTests/FlatIndexSearchTests.swift:577-594",
     "queries": [[0, 0, 0, 0]], "database": [[3, 4, 0, 0]], "k": 1, "ids": [[0]], "values": [[25.0]],
     "tol": 1e-3},
    {"kind": "knn", "metric": "l2", "source": "Tests/VectorAccelerateTests/FlatIndexSearchTests.swift:597-610",
     "queries": [[0, 0, 0, 0]], "database": [[1, 2, 3, 4]], "k": 1, "ids": [[0]], "values": [[30.0]],
     "tol": 1e-3},
    {"kind": "knn", "metric": "l2", "source": "Tests/VectorAccelerateTests/FlatIndexSearchTests.swift:613-626",
     "queries": [[4, 6, 8]], "database": [[1, 2, 3]], "k": 1, "ids": [[0]], "values": [[50.0]], "tol": 1e-3},
    {"kind": "knn", "metric": "l2", "source": "Tests/VectorAccelerateTests/FlatIndexSearchTests.swift:629-641",
     "queries": [[1.5, 2.5, 3.5, 4.5]], "database": [[1.5, 2.5, 3.5, 4.5]], "k": 1, "ids": [[0]],
     "values": [[0.0]], "tol": 1e-4},
    # ---------------------------------------------------------------- top-K selection
    {"kind": "topk", "mode": "min", "source": "Tests/VectorAccelerateTests/KernelTests.swift:621-643",
     "values_in": [[5, 2, 8, 1, 9, 3], [7, 4, 0.5, 6, 2.5, 1.5]], "k": 3,
     "ids": [[3, 1, 5], [2, 5, 4]], "values": [[1, 2, 3], [0.5, 1.5, 2.5]], "tol": 1e-5},
    {"kind": "topk", "mode": "max", "source": "Tests/VectorAccelerateTests/KernelTests.swift:645-659",
     "values_in": [[5, 2, 8, 1, 9, 3]], "k": 3, "ids": [[4, 2, 0]], "values": [[9, 8, 5]], "tol": 1e-5},
    {"kind": "topk", "mode": "min", "source": "Tests/VectorAccelerateTests/KernelTests.swift:661-672",
     "values_in": [list(range(100))], "k": 5, "ids": [[0, 1, 2, 3, 4]], "values": [[0, 1, 2, 3, 4]],
     "tol": 1e-5},
    {"kind": "topk", "mode": "min", "source": "Tests/VectorAccelerateTests/KernelTests.swift:676-681",
     "values_in": [[3, 1, 2]], "k": 3, "ids": [[1, 2, 0]], "values": [[1, 2, 3]], "tol": 1e-5},
    # k > n: the valid prefix is returned and the rest is padded (SearchAndRetrieval.metal:151-155)
    {"kind": "topk", "mode": "min", "source": "Tests/VectorAccelerateTests/KernelTests.swift:683-691",
     "values_in": [[3, 1, 2]], "k": 10, "ids": [[1, 2, 0] + [4294967295] * 7],
     "values": [[1, 2, 3] + ["inf"] * 7], "tol": 1e-5},
    # ---------------------------------------------------------------- binary / Hamming
    {"kind": "hamming_pairs", "source": "Tests/VectorAccelerateTests/KernelTests.swift:1936-1953",
     "vectors": [[1, 1, 1, 1], [1, 1, 1, 1]], "query": 0, "distances": [0, 0]},
    {"kind": "hamming_pairs", "source": "Tests/VectorAccelerateTests/KernelTests.swift:1955-1971",
     "vectors": [[1, 1, 1, 1], [-1, -1, -1, -1]], "query": 0, "distances": [0, 4]},
    {"kind": "hamming_pairs", "source": "Tests/VectorAccelerateTests/KernelTests.swift:1973-1986",
     "vectors": [[1, 1, -1, -1], [1, -1, 1, -1]], "query": 0, "distances": [0, 2]},
    {"kind": "hamming_matrix", "source": "Tests/VectorAccelerateTests/KernelTests.swift:3473-3494",
     "queries_bits": [[1, 0], [0, 1]], "database_bits": [[1, 0], [0, 0], [1, 1]],
     "row0": [0, 1, 1]},
    {"kind": "pack_bits", "source": "Tests/VectorAccelerateTests/KernelTests.swift:3496-3503",
     "bits": [1, 0, 1, 0, 0, 0, 0, 0], "words": [5]},
    {"kind": "pack_bits", "source": "Tests/VectorAccelerateTests/KernelTests.swift:3505-3512",
     "bits": [1] * 64, "words": [4294967295, 4294967295]},
    # ---------------------------------------------------------------- scalar quantization
    {"kind": "sq_roundtrip", "bits": 8, "source": "Tests/VectorAccelerateTests/KernelTests.swift:1775-1788",
     "data": [0.0, 0.25, 0.5, 0.75, 1.0, -0.25, -0.5, -0.75, -1.0], "tol": 0.02},
    {"kind": "sq_roundtrip", "bits": 4, "source": "Tests/VectorAccelerateTests/KernelTests.swift:1813-1827",
     "data": [0.0, 0.5, 1.0, -0.5, -1.0, 0.25, -0.25, 0.75], "tol": 0.2},
    {"kind": "sq_order", "bits": 8, "source": "Tests/VectorAccelerateTests/KernelTests.swift:1850-1862",
     "data": [-1000, -100, 0, 100, 1000]},
    # ---------------------------------------------------------------- parameter validation
    {"kind": "validate", "source": "Tests/VectorAccelerateTests/KernelTests.swift:956-973",
     "params": {"numQueries": 1, "numDataset": 100, "dimension": "maxDimension+1", "k": 8},
     "message_contains": ["dimension", "maxDimension"]},
    {"kind": "validate", "source": "Tests/VectorAccelerateTests/KernelTests.swift:975-991",
     "params": {"numQueries": 1, "numDataset": 100, "dimension": 768, "k": "maxK+1"},
     "message_contains": ["k", "maxK"]},
    {"kind": "validate", "source": "Tests/VectorAccelerateTests/KernelTests.swift:993-1046",
     "params": {"numQueries": 0, "numDataset": 100, "dimension": 768, "k": 8},
     "message_contains": ["numQueries"]},
    {"kind": "validate", "source": "Tests/VectorAccelerateTests/KernelTests.swift:993-1046",
     "params": {"numQueries": 1, "numDataset": 0, "dimension": 768, "k": 8},
     "message_contains": ["numDataset"]},
    {"kind": "validate", "source": "Tests/VectorAccelerateTests/KernelTests.swift:993-1046",
     "params": {"numQueries": 1, "numDataset": 100, "dimension": 0, "k": 8},
     "message_contains": ["dimension"]},
    {"kind": "validate", "source": "Tests/VectorAccelerateTests/KernelTests.swift:993-1046",
     "params": {"numQueries": 1, "numDataset": 100, "dimension": 768, "k": 0},
     "message_contains": ["k"]},
]


def main() -> None:
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "known_answers.json")
    with open(out, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "cases": CASES}, f, indent=1)
    print(f"wrote {len(CASES)} cases to {out}")


if __name__ == "__main__":
    main()
