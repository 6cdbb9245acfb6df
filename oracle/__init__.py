"""CPU oracle for the parity tests (test infrastructure, never on the product path)."""

from .hotpath import *  # noqa: F401,F403
