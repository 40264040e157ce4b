"""Plugin loader by directory name.  A plugin whose contract major is unknown is rejected at
load time without being used (reference tempo/plugins/registry.py:41-64); every MEASURED rate
is validated (card state present, zero foreign processes; registry.py:67-76)."""
from __future__ import annotations

import importlib
import pkgutil

from . import base
from .base import ContractError

_CACHE: dict = {}
_PKG = __name__.rsplit(".", 1)[0]


def available() -> list:
    pkg = importlib.import_module(_PKG)
    return sorted(m.name for m in pkgutil.iter_modules(pkg.__path__) if m.ispkg)


def _major(contract: str) -> str:
    parts = contract.rsplit("/", 1)
    return parts[0] if len(parts) == 2 else contract


def load(arch: str):
    if arch in _CACHE:
        return _CACHE[arch]
    try:
        mod = importlib.import_module(f"{_PKG}.{arch}")
    except ImportError as e:
        raise ContractError(f"plugin {arch!r} not found; known: {', '.join(available())}") from e
    if not hasattr(mod, "load"):
        raise ContractError(f"plugin {arch!r} declares no load()")
    p = mod.load()
    contract = getattr(p, "contract", None)
    if contract is None:
        raise ContractError(f"plugin {arch!r} declares no contract")
    if _major(contract) != base.CONTRACT_MAJOR:
        raise ContractError(f"plugin {arch!r} declares contract {contract!r}; the pipeline "
                            f"understands major {base.CONTRACT_MAJOR!r} only")
    _validate_rates(p, arch)
    _CACHE[arch] = p
    return p


def _validate_rates(p, arch: str) -> None:
    try:
        table = p.machine.symbols()
    except Exception as e:
        raise ContractError(f"plugin {arch!r}: symbols() failed: {e}") from e
    for sym, r in table.items():
        if not isinstance(r, base.Rate):
            raise ContractError(f"plugin {arch!r}: rate {sym!r} is not a Rate")
        r.check()


def by_arch_id(arch_id: str):
    """Find a plugin by its declared arch id (e.g. "sm_100a"), not by directory name."""
    for name in available():
        try:
            p = load(name)
        except ContractError:
            continue
        if getattr(p, "id", None) == arch_id:
            return p
    raise ContractError(f"no plugin with arch id {arch_id!r}")


def clear_cache() -> None:
    _CACHE.clear()
