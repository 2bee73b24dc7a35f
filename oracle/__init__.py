"""Test infrastructure only: the CPU oracle that the CUDA path is checked against.

Nothing in the ``swvr_b200`` package imports this; see ``swvr_oracle.py`` for what it restates.
"""
from .swvr_oracle import *  # noqa: F401,F403
