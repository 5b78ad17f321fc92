"""Distributed runtime: process groups, FSDP and TP engines, NVLink peer-memory collectives (lazy)."""

from importlib import import_module

_SUB = ("dist", "fsdp", "tp", "symm", "status", "watchdog")


def __getattr__(name):
    if name in _SUB:
        return import_module(f"vlmrl.parallel.{name}")
    raise AttributeError(name)


__all__ = list(_SUB)
