"""evelyn_b200 -- a B200 (sm_100a) decode engine for Evelyn's token loop.

The public Python API mirrors the reference runtime (src/runtime.rs, src/remote.rs):
``Model``, ``Session``, ``Batch``, ``FfnBackend``, ``DenseFfn``, ``CaptureFfn``,
``RemoteAarnnFfn``, ``argmax``, ``log_prob``, ``validate_token_ids``. All compute
runs in the CUDA library ``libevelyn_b200.so`` behind the C ABI of
``include/evelyn.h``; importing a name that needs it loads it lazily and fails
loudly when it is not built.
"""
from .runtime import (Batch, CaptureFfn, Config, DenseFfn, EvelynError, FfnBackend, Model,  # noqa: F401
                      RemoteAarnnFfn, Session, argmax, log_prob, tp_unique_id, validate_token_ids)

__all__ = ["Batch", "CaptureFfn", "Config", "DenseFfn", "EvelynError", "FfnBackend", "Model", "RemoteAarnnFfn",
           "Session", "argmax", "log_prob", "tp_unique_id", "validate_token_ids"]
