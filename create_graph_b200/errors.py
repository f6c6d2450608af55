"""The one exception type of the contract checks.

Mirrors ``create_graph.errors.ContractError`` (src/create_graph/errors.py:1-2):
a RuntimeError subclass, so code that catches RuntimeError keeps working.
"""


class ContractError(RuntimeError):
    """A model, a region or a registered fused op breaks a rule that
    create_graph relies on (one region per differentiated output, no gradient
    taken inside the model, no scaling after the region, ...)."""


class NativeError(RuntimeError):
    """The sm_100a library refused a call (bad shape, stride, size) or a CUDA
    launch failed. The message is the library's own."""
