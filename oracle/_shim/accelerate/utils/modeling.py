"""Stand-in for accelerate.utils.modeling (test infrastructure only)."""


def set_module_tensor_to_device(*args, **kwargs):
    raise NotImplementedError("accelerate is not installed; the oracle shim does not stream weights")
