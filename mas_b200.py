"""Import alias: ``import mas_b200`` loads the package directory ``mini-agent-serve_b200``.

A directory name with hyphens cannot appear in an import statement, so this module imports it by
name and puts the package itself in its place in sys.modules.
"""
import importlib
import sys

sys.modules[__name__] = importlib.import_module("mini-agent-serve_b200")
