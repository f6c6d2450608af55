"""
create_graph_b200: the conservative-force MLIP training step of create_graph,
with the region's forward, its dE/dx pass and the parameter backward through
that force running as hand-written sm_100a kernels.

    import create_graph_b200 as cg

    out, grads = cg.create_graph(model, data, outputs="energy", inputs=("pos",))
    loss = loss_fn(out, -grads["pos"])
    loss.backward()

The Python API is that of create_graph (src/create_graph/__init__.py:18-36):
``cg.compile`` marks the energy network, ``cg.create_graph`` runs the model
once and returns the output with its input gradients, ``cg.CompileConfig``
carries ``memory_budget`` and ``checkpoint``, and ``cg.custom_op`` registers a
fused op as forward1 / backward1 / backward2. The kernels live in one C-ABI
shared library (``include/cg_b200.h``) loaded by ``create_graph_b200.native``;
the fused ops of the energy network are in ``create_graph_b200.nn``.
"""

from create_graph_b200 import library, testing  # noqa: F401  (library: the torch.library operators)
from create_graph_b200.api import compile, create_graph, reset
from create_graph_b200.compile_config import CompileConfig, supports_in_graph_grad
from create_graph_b200.errors import ContractError, NativeError
from create_graph_b200.ops import FusedOp, custom_op

__version__ = "0.1.0"

__all__ = [
    "CompileConfig",
    "ContractError",
    "FusedOp",
    "NativeError",
    "compile",
    "create_graph",
    "custom_op",
    "reset",
    "supports_in_graph_grad",
    "testing",
]
