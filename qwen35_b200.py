"""Import name of the framework package.

The package source lives in the directory
``qwen3.5-397b-mi300a-bespoke-vibesys-20260920_b200/`` next to this file. That name is not a
valid Python identifier, so this module stands in for it: setting ``__path__`` makes this
module a package whose submodules (``qwen35_b200.models``, ``qwen35_b200.ops``, ...) are
looked up in that directory.
"""

from __future__ import annotations

import os as _os

PACKAGE_DIR = _os.path.join(
    _os.path.dirname(_os.path.abspath(__file__)),
    "qwen3.5-397b-mi300a-bespoke-vibesys-20260920_b200",
)
__path__ = [PACKAGE_DIR]
__version__ = "0.1.0"

_init = _os.path.join(PACKAGE_DIR, "__init__.py")
if _os.path.exists(_init):
    with open(_init) as _f:
        exec(compile(_f.read(), _init, "exec"))
