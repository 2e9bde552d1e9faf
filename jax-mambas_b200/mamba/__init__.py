"""B200 (sm_100a) selective scan behind the JAX-Mambas op interface."""
from .selective_scan_cuda import (  # noqa: F401
    register_cuda_kernel,
    selective_scan,
    selective_scan_fn,
    selective_scan_reference,
    selective_state_update,
)
