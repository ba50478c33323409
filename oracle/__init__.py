"""Parity oracle for the HdcMamba-9v3 layer forward -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this directory.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and its
``--impl reference`` arm) use it, and only as the checker or as the timed CPU
baseline -- never as the thing that is measured or shipped.

``oracle.restate`` is a vectorised PyTorch-CPU restatement of the reference
forward (``hdcmamba/model.py`` of N01N9/hdcmamba).  It reproduces every
rounding point and every launch-argument quirk of the shipped kernels, and it
is pinned against golden vectors that were produced by running the unmodified
reference under ``TRITON_INTERPRET=1`` (``tests/golden/make_golden.py``).
"""
from .restate import *  # noqa: F401,F403
