"""Import alias: ``import mas_b200`` loads the package directory ``mini-agent-serve_b200`` as ``mas_b200``.

A directory name with hyphens cannot appear in an import statement, so this module loads the package
from its directory under the name ``mas_b200`` and puts it in its own place in sys.modules. Its
submodules are then ``mas_b200.ops``, ``mas_b200.workloads`` and so on, one module object each.
"""
import importlib.util
import sys
from pathlib import Path

_pkg_dir = Path(__file__).resolve().parent / "mini-agent-serve_b200"
_spec = importlib.util.spec_from_file_location(__name__, _pkg_dir / "__init__.py",
                                               submodule_search_locations=[str(_pkg_dir)])
_pkg = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _pkg
_spec.loader.exec_module(_pkg)
