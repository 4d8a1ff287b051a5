"""Loader for the golden fixtures in tests/golden/ (made by the reference's
own code; see tests/golden/make_golden.py)."""
from __future__ import annotations

import dataclasses
import functools
import json
import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


@dataclasses.dataclass
class Enc:
    """Plain container with the reference ChunkedEncoded fields
    (afterimage/runtime/huffman_chunked.py:135-148)."""
    packed: np.ndarray
    chunk_offsets: np.ndarray
    chunk_nbytes: np.ndarray
    sym_lut: np.ndarray
    len_lut: np.ndarray
    max_bits: int
    chunk_size: int
    n_symbols: int
    shape: tuple

    @property
    def n_chunks(self) -> int:
        return len(self.chunk_offsets)


@functools.lru_cache(maxsize=1)
def manifest() -> dict:
    return json.loads((GOLDEN / "manifest.json").read_text())


@functools.lru_cache(maxsize=1)
def _npz():
    with np.load(GOLDEN / "cases.npz") as z:
        return {k: z[k] for k in z.files}


def cases(kind: str | None = None) -> list[dict]:
    return [c for c in manifest()["cases"] if kind is None or c["kind"] == kind]


def case(name: str) -> dict:
    for c in manifest()["cases"]:
        if c["name"] == name:
            return c
    raise KeyError(name)


def arr(name: str, field: str) -> np.ndarray:
    return _npz()[f"{name}/{field}"]


def has(name: str, field: str) -> bool:
    return f"{name}/{field}" in _npz()


def enc(name: str) -> Enc:
    c = case(name)
    return Enc(packed=arr(name, "packed"), chunk_offsets=arr(name, "chunk_offsets"),
               chunk_nbytes=arr(name, "chunk_nbytes"), sym_lut=arr(name, "sym_lut"),
               len_lut=arr(name, "len_lut"), max_bits=c["max_bits"],
               chunk_size=c["chunk_size"], n_symbols=c["n_symbols"],
               shape=tuple(c["enc_shape"]))
