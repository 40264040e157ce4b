"""Plugin discovery and admission.

A plugin is a sub-package of ``tempo.plugins`` whose ``load()`` returns the plugin object.  The
admission rules are the contract's (the reference applies them in tempo/plugins/registry.py:
41-88): a plugin that declares a contract of another major version is refused before any of
it is used, and every rate in its machine table must pass ``Rate.check`` (a MEASURED rate needs
its card state and a clean card).  Admission runs as a sequence of checks over the imported
module (``_ADMISSION``); the first one that fails raises ContractError.  Admitted plugins are
cached by directory name.
"""
from __future__ import annotations

import importlib
import pkgutil

from . import base
from .base import ContractError

_PKG = __name__.rpartition(".")[0]
_admitted: dict = {}


def available() -> list:
    """Directory names of every plugin package, sorted."""
    root = importlib.import_module(_PKG)
    return sorted(info.name for info in pkgutil.iter_modules(root.__path__) if info.ispkg)


def _contract_family(contract: str) -> str:
    """'tempo/arch/1' -> 'tempo/arch' (the part a plugin and the pipeline must share)."""
    family, sep, _version = contract.rpartition("/")
    return family if sep else contract


def _has_loader(arch, module, plugin):
    if not callable(getattr(module, "load", None)):
        raise ContractError(f"plugin package {arch!r} has no load() function")


def _declares_known_contract(arch, module, plugin):
    contract = getattr(plugin, "contract", None)
    if not contract:
        raise ContractError(f"plugin {arch!r} does not say which contract it implements")
    if _contract_family(contract) != base.CONTRACT_MAJOR:
        raise ContractError(f"plugin {arch!r} implements {contract!r}; this pipeline speaks "
                            f"{base.CONTRACT_MAJOR!r} only, so the plugin is not used")


def _rates_are_admissible(arch, module, plugin):
    try:
        symbols = plugin.machine.symbols()
    except Exception as e:
        raise ContractError(f"plugin {arch!r}: its machine table could not be listed ({e})") from e
    for sym, rate in symbols.items():
        if not isinstance(rate, base.Rate):
            raise ContractError(f"plugin {arch!r}: symbol {sym!r} is a "
                                f"{type(rate).__name__}, not a Rate")
        rate.check()


# _has_loader runs before load() is called; the others on the loaded plugin
_ADMISSION = (_declares_known_contract, _rates_are_admissible)


def load(arch: str):
    """The admitted plugin in package ``arch`` (cached), or ContractError."""
    if arch in _admitted:
        return _admitted[arch]
    try:
        module = importlib.import_module(f"{_PKG}.{arch}")
    except ImportError as e:
        raise ContractError(f"no plugin package {arch!r} (available: "
                            f"{', '.join(available())})") from e
    _has_loader(arch, module, None)
    plugin = module.load()
    for check in _ADMISSION:
        check(arch, module, plugin)
    _admitted[arch] = plugin
    return plugin


def by_arch_id(arch_id: str):
    """The admitted plugin whose declared ``id`` is ``arch_id`` (e.g. "sm_100a")."""
    for name in available():
        try:
            plugin = load(name)
        except ContractError:
            continue
        if getattr(plugin, "id", None) == arch_id:
            return plugin
    raise ContractError(f"no admitted plugin declares arch id {arch_id!r}")


def clear_cache() -> None:
    _admitted.clear()
