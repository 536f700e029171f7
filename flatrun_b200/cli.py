"""``flatrun`` with ``--backend cuda``: the reference command line, unchanged,
with the B200 backend selectable.

    python -m flatrun_b200.cli run <model.gguf> --prompt "..." --backend cuda
    python -m flatrun_b200.cli serve <model.gguf> --backend cuda

The reference CLI offers ``--backend {python,native}`` (src/flatrun/cli.py:
1032-1042) and hands the choice to ``get_backend`` (cli.py:1610) and then to
``make_qwen2_forwarder``.  This launcher, without editing the reference:

* registers the CUDA backend (``integration.register``) and maps the name
  ``"cuda"`` to the adapter that answers ``name == "native"``, the spelling
  the forwarder's dispatch gate checks (qwen2.py:1466, :2250);
* adds Q5_K and Q1_0 to the forwarder's quant -> method table
  (``integration.extend_forwarder_method_table``);
* adds ``"cuda"`` to the choices of every ``--backend`` option the reference
  parser declares, then runs the reference's own ``flatrun.cli.main``.
"""

from __future__ import annotations

import argparse
import sys
from contextlib import contextmanager

from . import integration


@contextmanager
def backend_choice_added(name: str = "cuda"):
    """While active, an argparse option ``--backend`` declared with the
    reference's choices also accepts `name`."""
    orig = argparse._ActionsContainer.add_argument

    def add_argument(self, *args, **kwargs):
        choices = kwargs.get("choices")
        if "--backend" in args and choices is not None and "native" in choices and name not in choices:
            kwargs = dict(kwargs, choices=list(choices) + [name])
        return orig(self, *args, **kwargs)

    argparse._ActionsContainer.add_argument = add_argument
    try:
        yield
    finally:
        argparse._ActionsContainer.add_argument = orig


def install(backend_module=None, qwen2_module=None) -> type:
    """Register the backends and return the class ``get_backend("cuda")``
    now builds (the CUDA backend under the forwarder's ``native`` name)."""
    if backend_module is None:
        from flatrun.runtime import backend as backend_module  # type: ignore[import-not-found]
    _, adapter = integration.register(backend_module)
    backend_module._BACKENDS["cuda"] = adapter
    integration.extend_forwarder_method_table(qwen2_module)
    return adapter


def main(argv: list[str] | None = None) -> int:
    install()
    with backend_choice_added("cuda"):
        from flatrun.cli import main as reference_main  # type: ignore[import-not-found]
        return reference_main(argv)


if __name__ == "__main__":
    sys.exit(main())
