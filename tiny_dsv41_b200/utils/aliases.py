"""Import hook that serves modules of this library under the module paths of the original
packages (``dsv41_train.*``, ``rollout_manager.*``), for drop-in imports.

``install(package, table)`` answers ``import <package>.<key>`` for every key of ``table`` by
importing ``table[key]`` and registering that module object under both names.
"""

from __future__ import annotations

import importlib
import importlib.abc
import importlib.util
import sys


class AliasFinder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    def __init__(self, package: str, table: dict[str, str]) -> None:
        self.package = package
        self.table = dict(table)

    def _target(self, fullname: str) -> str | None:
        prefix = self.package + "."
        return self.table.get(fullname[len(prefix):]) if fullname.startswith(prefix) else None

    def find_spec(self, fullname, path=None, target=None):
        if self._target(fullname) is None:
            return None
        return importlib.util.spec_from_loader(fullname, self)

    def create_module(self, spec):
        module = importlib.import_module(self._target(spec.name))
        sys.modules[spec.name] = module
        return module

    def exec_module(self, module):  # the target module has already run
        return None


def install(package: str, table: dict[str, str]) -> AliasFinder:
    for finder in sys.meta_path:
        if isinstance(finder, AliasFinder) and finder.package == package:
            finder.table.update(table)
            return finder
    finder = AliasFinder(package, table)
    sys.meta_path.insert(0, finder)  # ahead of the path finder, which would load a second copy
    return finder
