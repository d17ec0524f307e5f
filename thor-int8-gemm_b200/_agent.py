"""Start-up plumbing shared by the package's two comfy patches (`patch_int8`, `fused_patch`).

Both patches are installed by one `.pth` line when the interpreter starts, so each of them
has to: pick its mode from an environment variable or a mode file, refuse a comfy-kitchen
release it was not validated against, report on stderr under its own tag, never raise, and
apply itself to its target module as soon as that module has finished importing -- or at
once, when it already has.  This module implements those mechanics once.

Applying a patch on import: a meta-path finder (`ImportHook`, one per patch) is consulted
before the normal finders; for a module it watches, it asks the standard path finder for
the spec and puts a small loader (`_ThenPatch`) in front of the real one.  That loader
hands the module back to the real loader (and restores it on the module's spec, so nothing
of the hook stays visible afterwards), executes it, then runs the patch callback.
"""
from __future__ import annotations

import importlib.abc
import importlib.machinery
import os
import sys
from typing import Callable, Dict, Mapping, Optional


def say(tag: str, message: str) -> None:
    """One tagged line on stderr, flushed (start-up logs of a long-running server)."""
    print(f"{tag} {message}", file=sys.stderr, flush=True)


def read_mode(env_name: str, mode_file: str, aliases: Optional[Mapping[str, str]] = None) -> str:
    """The patch's mode: the environment variable when it is set and not empty, else the
    contents of `mode_file` (empty or unreadable: "off"); lower-cased with surrounding
    blanks dropped, then mapped through `aliases` (e.g. "1" -> "on")."""
    raw = os.environ.get(env_name)
    if raw:
        value = raw.strip().lower()
    else:
        try:
            with open(mode_file) as fh:
                value = fh.read().strip().lower() or "off"
        except OSError:
            value = "off"
    return (aliases or {}).get(value, value)


def kitchen_version() -> Optional[str]:
    """The installed comfy-kitchen distribution's version, or None when it is absent."""
    try:
        from importlib.metadata import version
        return version("comfy-kitchen")
    except Exception:
        return None


class _ThenPatch(importlib.abc.Loader):
    """Loader placed in front of a watched module's real loader for one import."""

    def __init__(self, real: importlib.abc.Loader, patch: Callable[[object], None]):
        self._real = real
        self._patch = patch

    def create_module(self, spec):
        return self._real.create_module(spec)

    def exec_module(self, module):
        spec = getattr(module, "__spec__", None)
        if spec is not None and spec.loader is self:
            spec.loader = self._real
        if getattr(module, "__loader__", None) is self:
            module.__loader__ = self._real
        self._real.exec_module(module)
        self._patch(module)

    def __getattr__(self, name):        # get_code, get_source, resource readers, ...
        return getattr(self._real, name)


class ImportHook(importlib.abc.MetaPathFinder):
    """Meta-path finder of one patch (`owner`): module name -> callback run right after that
    module executes."""

    def __init__(self, owner: str, targets: Dict[str, Callable[[object], None]]):
        self.owner = owner
        self.targets = dict(targets)

    def find_spec(self, name, path, target=None):
        patch = self.targets.get(name)
        if patch is None:
            return None
        spec = importlib.machinery.PathFinder.find_spec(name, path)
        if spec is None or spec.loader is None:
            return None
        spec.loader = _ThenPatch(spec.loader, patch)
        return spec


def when_imported(owner: str, targets: Dict[str, Callable[[object], None]]) -> None:
    """Run targets[name](module) for each module now if it is already imported, and when it
    is imported otherwise.  A later call by the same owner replaces its earlier hook."""
    pending = {}
    for name, patch in targets.items():
        module = sys.modules.get(name)
        if module is not None:
            patch(module)
        else:
            pending[name] = patch
    sys.meta_path[:] = [f for f in sys.meta_path if not (isinstance(f, ImportHook) and f.owner == owner)]
    if pending:
        sys.meta_path.insert(0, ImportHook(owner, pending))
