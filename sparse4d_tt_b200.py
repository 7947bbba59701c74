"""Import name of the package that lives in the directory ``sparse4d-tt_b200/``.

A hyphen cannot appear in a Python import, so this module loads
``sparse4d-tt_b200/__init__.py`` as the package ``sparse4d_tt_b200`` and puts it in
``sys.modules`` in its own place.  ``import sparse4d_tt_b200`` and
``from sparse4d_tt_b200.dfa import DeformableFeatureAggregation`` then work from the
repository root.
"""
import importlib.util as _ilu
import os as _os
import sys as _sys

_PKG_DIR = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "sparse4d-tt_b200")
_spec = _ilu.spec_from_file_location(
    __name__, _os.path.join(_PKG_DIR, "__init__.py"), submodule_search_locations=[_PKG_DIR]
)
_mod = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
