"""Import name of the package kept in ``flashvsr-optimizations_b200/``.

The directory name is not a Python identifier, so this module loads the
package from it and takes its place in ``sys.modules``:
``import flashvsr_optimizations_b200`` gives the package, and its submodules
(``flashvsr_optimizations_b200.ops`` ...) resolve from that directory.
"""
import importlib.util as _ilu
import os as _os
import sys as _sys

_DIR = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "flashvsr-optimizations_b200")
_spec = _ilu.spec_from_file_location(__name__, _os.path.join(_DIR, "__init__.py"),
                                     submodule_search_locations=[_DIR])
_mod = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
