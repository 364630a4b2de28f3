"""Import shim: `import drama3_b200` loads the package in the `drama-3-tr_b200/` directory (a
directory name with hyphens cannot be imported directly)."""

import importlib.util
import sys
from pathlib import Path

_DIR = Path(__file__).resolve().parent / "drama-3-tr_b200"
_spec = importlib.util.spec_from_file_location("drama3_b200", _DIR / "__init__.py", submodule_search_locations=[str(_DIR)])
_mod = importlib.util.module_from_spec(_spec)
sys.modules["drama3_b200"] = _mod
_spec.loader.exec_module(_mod)
