"""Import alias for the package directory ``agillm4.1_b200/``.

A directory name containing a dot cannot be imported with a plain ``import``
statement, so this module loads ``agillm4.1_b200/__init__.py`` as the package
``agillm41_b200`` (submodules resolve inside that directory) and replaces
itself with it in ``sys.modules``.
"""
import importlib.util
import os
import sys

_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "agillm4.1_b200")
_spec = importlib.util.spec_from_file_location(__name__, os.path.join(_DIR, "__init__.py"),
                                               submodule_search_locations=[_DIR])
_pkg = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _pkg
_spec.loader.exec_module(_pkg)
