"""The backend seam record for the fusion-template groups.

The reference keys every specialization by the backend's fingerprint and
describes a backend by a capability record, ``pdum.dsl.registry.Backend(name,
render, compile, fp, ...)`` (``packages/dsl/src/pdum/dsl/registry.py:56-70``,
``register_backend`` at ``:119``).  ``b200_backend()`` returns that record
for this library:

* ``fp = ("b200_sm100a", <pdb_version()>)`` -- a library change is a new key;
* ``render(region, plan=None, backend=None)`` recognises the region and
  returns the launch it maps to (entry point and its arguments) as text --
  the "source" of a prebuilt-kernel backend;
* ``compile(source, name)`` returns the ``compile_tile`` runner of that
  rendered region (numpy in / out, ``run_t`` for device tensors).

It serves fusion-template groups only (flash, row reductions, contraction
epilogue, map chain) and refuses everything else with ``Untranslatable``;
there is no dispatch to other backends.  Requires the reference DSL.
"""

from __future__ import annotations

_RENDERED: dict[str, object] = {}  # rendered source -> region (compile looks the region up)


def _render(region, plan=None, backend=None):
    from .tile import compile_tile

    run = compile_tile(region)  # recognises the template or raises Untranslatable
    key = region.key.hex() if isinstance(getattr(region, "key", None), bytes) else str(id(region))
    source = f"// sm100a {run.source}\n// region {key}"
    _RENDERED[source] = region
    return source


def _compile(source, name=None):
    from .tile import compile_tile

    region = _RENDERED.get(source)
    if region is None:
        raise KeyError("source was not rendered by this backend")
    return compile_tile(region)


def b200_backend():
    """The ``pdum.dsl.registry.Backend`` record of this library."""
    from pdum.dsl.registry import Backend

    from ._lib import version

    return Backend(name="b200_sm100a", render=_render, compile=_compile, fp=("b200_sm100a", version()))
