"""``ops.ttt_linear`` / ``ops.ttt_mlp`` with the reference's signatures (ops/__init__.py:1-2),
computed by the sm_100a kernels (forward and backward) instead of a Python scan."""

from ops.ttt_linear import ttt_linear  # noqa: F401
from ops.ttt_mlp import ttt_mlp  # noqa: F401
