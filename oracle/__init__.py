"""CPU oracle for the Mamba-Integer hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the CPU legs of ``bench.py`` as the checker / CPU baseline.  The product path
(``mamba_integer_b200``) never imports this package.

``oracle.lib`` wraps ``libmi_oracle.so`` (``mi_oracle.c``), a C restatement of
each stage of the reference CPU path in the reference's own floating-point
order; ``oracle.model`` strings those stages together exactly as
``MambaIntegerModel.forward`` does (src/mamba_integer_model.py:486-495).
"""
from . import lib  # noqa: F401
