"""Pickle checkpoint I/O in the reference's on-disk format.

Format (reference ``utils/checkpoint.py:19-98``): ``pickle.dumps(dict)`` where the
dict holds every attribute assigned on the ``Checkpoint`` object (values with a
``save()`` method are serialised through it) plus ``"_timestamp"``.  Writes go
through ``<file>.tmp`` and an atomic rename.  ``parallel=True`` serialises on a
single background thread (the previous write is awaited before the next one).

``gs://`` paths are rejected: this framework has no object-store client.
Sharded runs gather to rank 0 before calling ``save`` (single-file format);
``save_sharded`` / ``load_sharded`` are the per-rank fast path (one pickle per
rank plus an index), an addition with no counterpart in the reference.
"""

from __future__ import annotations

import concurrent.futures
import json
import os
import pickle
import time
from typing import Any, Dict, Optional, Sequence


class Checkpoint:
    def __init__(self, filename: Optional[str], parallel: bool = True):
        object.__setattr__(self, "_filename", filename)
        object.__setattr__(self, "_values", {})
        object.__setattr__(self, "_parallel", bool(parallel))
        object.__setattr__(self, "_pending", None)
        object.__setattr__(self, "_pool", concurrent.futures.ThreadPoolExecutor(1, "checkpoint") if parallel else None)

    def __setattr__(self, key: str, value: Any) -> None:
        if key.startswith("_"):
            object.__setattr__(self, key, value)
        else:
            self._values[key] = value

    def __getattr__(self, key: str) -> Any:
        if key.startswith("_"):
            raise AttributeError(key)
        try:
            return self._values[key]
        except KeyError as exc:
            raise AttributeError(key) from exc

    def set_model(self, model: Any) -> None:
        for key, val in vars(model).items():
            if hasattr(val, "save") or key == "config":
                self._values[key] = val

    # ------------------------------------------------------------------ save
    def _payload(self, keys: Optional[Sequence[str]]) -> bytes:
        keys = tuple(self._values if keys is None else keys)
        if any(k.startswith("_") for k in keys):
            raise ValueError(f"private keys cannot be saved: {keys}")
        data: Dict[str, Any] = {}
        for k in keys:
            v = self._values[k]
            data[k] = v if isinstance(v, dict) or not hasattr(v, "save") else v.save()
        data["_timestamp"] = time.time()
        return pickle.dumps(data, protocol=pickle.HIGHEST_PROTOCOL)

    @staticmethod
    def _write_atomic(filename: str, content: bytes) -> None:
        if filename.startswith("gs://"):
            raise NotImplementedError("gs:// checkpoints need an object-store client, which is not bundled")
        parent = os.path.dirname(filename) or "."
        os.makedirs(parent, exist_ok=True)
        tmp = os.path.join(parent, os.path.basename(filename) + ".tmp")
        with open(tmp, "wb") as fh:
            fh.write(content)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, filename)

    def save(self, filename: Optional[str] = None, keys: Optional[Sequence[str]] = None) -> None:
        target = filename or self._filename
        if not target:
            raise ValueError("no checkpoint filename given")
        content = self._payload(keys)  # snapshot synchronously; only the disk write is async
        if self._parallel:
            self.wait()
            object.__setattr__(self, "_pending", self._pool.submit(self._write_atomic, target, content))
        else:
            self._write_atomic(target, content)

    def wait(self) -> None:
        if self._pending is not None:
            self._pending.result()
            object.__setattr__(self, "_pending", None)

    # ------------------------------------------------------------------ load
    def load_as_dict(self, filename: Optional[str] = None) -> Dict[str, Any]:
        target = filename or self._filename
        if not target:
            raise ValueError("no checkpoint filename given")
        if target.startswith("gs://"):
            raise NotImplementedError("gs:// checkpoints need an object-store client, which is not bundled")
        with open(target, "rb") as fh:
            data = pickle.load(fh)
        if not isinstance(data, dict) or "_timestamp" not in data:
            raise ValueError(f"{target} is not a checkpoint pickle (missing _timestamp)")
        return data

    def load_model(self, model: Any, filename: Optional[str] = None) -> Any:
        data = self.load_as_dict(filename)
        updates = {k: getattr(model, k).load(v) for k, v in data.items() if k in vars(model) and k != "config"}
        return model.replace(**updates)


def save_sharded(directory: str, rank: int, world_size: int, payload: Dict[str, Any], step: int) -> str:
    """Per-rank shard file plus (rank 0) an index; no gather, no rank-0 bottleneck."""
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"shard_{rank:05d}_of_{world_size:05d}.pkl")
    Checkpoint._write_atomic(path, pickle.dumps({"payload": payload, "step": step, "_timestamp": time.time()},
                                                protocol=pickle.HIGHEST_PROTOCOL))
    if rank == 0:
        index = {"world_size": world_size, "step": step,
                 "shards": [f"shard_{r:05d}_of_{world_size:05d}.pkl" for r in range(world_size)]}
        Checkpoint._write_atomic(os.path.join(directory, "index.json"), json.dumps(index).encode())
    return path


def load_sharded(directory: str, rank: int) -> Dict[str, Any]:
    with open(os.path.join(directory, "index.json")) as fh:
        index = json.load(fh)
    with open(os.path.join(directory, index["shards"][rank]), "rb") as fh:
        return pickle.load(fh)


__all__ = ["Checkpoint", "save_sharded", "load_sharded"]
