"""Falsifier G2: a plugin with no capabilities.  Every section refuses structurally
(PluginCapabilityError / NotSupported), never with AttributeError."""
from __future__ import annotations

from ..base import CONTRACT, NotSupported, PluginCapabilityError, Report


class _Refuse:
    def __init__(self, section):
        self._section = section

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)

        def refuse(*a, **k):
            raise PluginCapabilityError(f"null plugin: {self._section}.{name} is not offered")
        return refuse


class _Machine(_Refuse):
    def __init__(self):
        super().__init__("machine")

    def arch(self):
        return "null"

    def symbols(self):
        return {}

    def channels(self):
        return {}


class NullPlugin:
    id = "null"
    contract = CONTRACT
    description = "falsifier: refuses everything structurally"

    def __init__(self):
        self.machine = _Machine()
        self.memory = _Refuse("memory")
        self.tensor = _Refuse("tensor")
        self.resources = _Refuse("resources")
        self.sync = _Refuse("sync")
        self.classifier = None
        self.skeletons = _Refuse("skeletons")
        self.toolchain = _Refuse("toolchain")
        self.meters = _Refuse("meters")

    def declared_stubs(self):
        return ("everything",)

    def selftest(self):
        r = Report(self.id)
        try:
            self.skeletons.variants(None)
            r.check("skeletons refuse structurally", False)
        except PluginCapabilityError:
            r.check("skeletons refuse structurally", True)
        except NotSupported:
            r.check("skeletons refuse structurally", True)
        return r


def load():
    return NullPlugin()
