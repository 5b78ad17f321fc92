"""Config-dict -> command-line flags (reference ``utils/configs.py:3-12``).

The reference registers one absl flag per entry of an ``ml_collections``
ConfigDict, typed from the default value.  ``define_flag_dict`` does the same
for a plain dict through ``absl.flags`` when absl is importable, and
``build_arg_parser`` offers the argparse equivalent (used by the CLIs so they
also accept ``--flag=value`` and ``--flag value``).  Aliases map alternative
spellings (``--lr`` for ``--learning_rate``) onto the same destination.
"""

from __future__ import annotations

import argparse
from typing import Any, Dict, Mapping, Optional


def define_flag_dict(config: Mapping[str, Any]):
    from absl import flags

    for key, val in config.items():
        if isinstance(val, bool):
            flags.DEFINE_bool(key, val, f"Configuration for {key}")
        elif isinstance(val, int):
            flags.DEFINE_integer(key, val, f"Configuration for {key}")
        elif isinstance(val, float):
            flags.DEFINE_float(key, val, f"Configuration for {key}")
        elif isinstance(val, str):
            flags.DEFINE_string(key, val, f"Configuration for {key}")
    return flags.FLAGS


def _str2bool(s: str) -> bool:
    if isinstance(s, bool):
        return s
    low = str(s).strip().lower()
    if low in ("1", "true", "yes", "y", "on"):
        return True
    if low in ("0", "false", "no", "n", "off"):
        return False
    raise argparse.ArgumentTypeError(f"not a boolean: {s!r}")


def build_arg_parser(config: Mapping[str, Any], aliases: Optional[Mapping[str, str]] = None,
                     description: str = "") -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description=description)
    alias_of: Dict[str, list] = {}
    for alt, dest in (aliases or {}).items():
        alias_of.setdefault(dest, []).append(alt)
    for key, val in config.items():
        names = [f"--{key}"] + [f"--{a}" for a in alias_of.get(key, [])]
        if isinstance(val, bool):
            parser.add_argument(*names, dest=key, type=_str2bool, nargs="?", const=True, default=val)
        elif isinstance(val, int):
            parser.add_argument(*names, dest=key, type=int, default=val)
        elif isinstance(val, float):
            parser.add_argument(*names, dest=key, type=float, default=val)
        else:
            parser.add_argument(*names, dest=key, type=str, default=val)
    return parser


__all__ = ["define_flag_dict", "build_arg_parser"]
