"""Import name for the package directory ``cti-inference-optimization_b200/``.

The directory name is not a Python identifier, so ``import cti_b200`` loads
it through this file: the package's ``__init__`` runs under the name
``cti_b200`` with the directory as its search path, and replaces this module
in ``sys.modules``.
"""
import importlib.util
import os
import sys

_PKG_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cti-inference-optimization_b200")
_spec = importlib.util.spec_from_file_location(
    __name__, os.path.join(_PKG_DIR, "__init__.py"), submodule_search_locations=[_PKG_DIR])
_mod = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
