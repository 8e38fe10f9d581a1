"""pytest plugin: run radiance's own NVFP4 test file against this package.

    python -m pytest -p tests.reference_alias -q baseline/_ref/tests/test_nvfp4.py

radiance's tests (tests/test_nvfp4.py in jamespa16/radiance) import ``from radiance import nvfp4``,
and its model code (src/radiance/model/transformer.py:10) does the same to convert ``nn.Linear``
layers into ``nvfp4.FP4Linear``.  This plugin puts the unmodified reference install
(``baseline/_ref``, or ``$RADIANCE_REF``) on ``sys.path`` for ``radiance.config`` and
``radiance.model``, and binds the module name ``radiance.nvfp4`` to ``radiance_b200.nvfp4`` before
anything imports it.  Every ``nvfp4.*`` the test file and the model touch then resolves to this
package: the format helpers to ``radiance_b200.nvfp4.reference``, ``quantize`` / ``mm`` /
``FP4Linear`` to the CUDA library.  radiance's own ``nvfp4`` package is never imported.

The plugin is test infrastructure only; nothing in ``radiance_b200`` imports it.
"""

from __future__ import annotations

import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_REF = os.environ.get("RADIANCE_REF", os.path.join(_ROOT, "baseline", "_ref"))


def _bind() -> None:
    if _ROOT not in sys.path:
        sys.path.insert(0, _ROOT)
    if not os.path.isdir(os.path.join(_REF, "radiance")):
        raise RuntimeError(f"reference_alias: no radiance package under {_REF} (set RADIANCE_REF)")
    if _REF not in sys.path:
        sys.path.append(_REF)
    import radiance_b200.nvfp4 as ours

    if "radiance.nvfp4" in sys.modules and sys.modules["radiance.nvfp4"] is not ours:
        raise RuntimeError("reference_alias: radiance.nvfp4 was imported before the alias was bound")
    sys.modules["radiance.nvfp4"] = ours
    import radiance

    radiance.nvfp4 = ours


_bind()


def pytest_report_header(config):
    import radiance_b200.nvfp4 as ours

    return [f"radiance.nvfp4 -> {ours.__name__} ({os.path.dirname(ours.__file__)}); "
            f"radiance.config / radiance.model from {_REF}"]
