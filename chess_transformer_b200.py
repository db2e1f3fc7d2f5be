"""Import shim: the package lives in the directory `chess-transformer_b200/`, whose name is not a Python identifier.

`import chess_transformer_b200` loads that directory as the package `chess_transformer_b200` (its submodules import
normally from then on).
"""
import importlib.util
import sys
from pathlib import Path

_DIRECTORY = Path(__file__).resolve().parent / "chess-transformer_b200"
_spec = importlib.util.spec_from_file_location(__name__, _DIRECTORY / "__init__.py", submodule_search_locations=[str(_DIRECTORY)])
_package = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _package
_spec.loader.exec_module(_package)
