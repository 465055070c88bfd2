"""Import shim: the package lives in the directory ``im-not-llm_b200/`` (a name
Python cannot import directly); ``import im_not_llm_b200`` loads it from there."""
import importlib.util as _u
import sys as _sys
from pathlib import Path as _Path

_dir = _Path(__file__).resolve().with_name("im-not-llm_b200")
_spec = _u.spec_from_file_location(__name__, _dir / "__init__.py", submodule_search_locations=[str(_dir)])
_mod = _u.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
