"""Drop-in import name: ``import dot`` gives the dot_b200 implementation with
the reference package's public surface (``dot/__init__.py:32-64`` of
caseysm/dot)."""

from dot_b200 import *  # noqa: F401,F403
from dot_b200 import __all__  # noqa: F401

from . import _ops  # noqa: F401,E402
