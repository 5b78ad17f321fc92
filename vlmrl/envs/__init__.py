"""Environments: ``BaseEnv`` protocol, registry and built-in tasks (reference ``envs/__init__.py``)."""

from vlmrl.envs.base import BaseEnv, BaseState, create_env, register_env

__all__ = ["BaseEnv", "BaseState", "create_env", "register_env"]
