"""sdcguard_b200: a Blackwell-native (sm_100a) guard against silent data corruption in LLM serving and training.

Every checked hot path is a hand-written sm_100a CUDA kernel that fuses its check into the work it guards
(checked GEMMs with ABFT epilogues, checksummed KV-block transfer, checksummed all-to-all, sampled attention
recompute). The Python layer keeps the `sdcguard` CLI, the checksum-record schema and the offline coverage gate.
"""
__version__ = "0.1.0"

# The reference's top-level names, imported on first use (commands that need no PyTorch start at once):
#   SDCGuard / SDCError (training guard), Canary, check_replicas / weight_fingerprint (data-parallel votes),
#   ServeGuard (+ ServeGuard.attach for any model), check_matmul / check_linear / CheckResult (a product computed
#   elsewhere), EventLog / SDCEvent / rollback_checkpoint, FaultInjector / FaultModel / corrupt_ (fault injection)
_LAZY = {
    "Canary": "train.canary", "CheckResult": "numerics.check", "check_linear": "numerics.check",
    "check_matmul": "numerics.check", "EventLog": "utils.events", "SDCEvent": "utils.events",
    "rollback_checkpoint": "utils.events", "SDCError": "train.guard", "SDCGuard": "train.guard",
    "FaultInjector": "utils.inject", "FaultModel": "utils.inject", "corrupt_": "utils.inject",
    "check_replicas": "train.replica", "weight_fingerprint": "train.replica", "ServeGuard": "serve.attach",
    "attach": "serve.attach", "DispatchGuard": "train.dispatch",
}
__all__ = list(_LAZY)


def __getattr__(name):
    if name in _LAZY:
        import importlib
        value = getattr(importlib.import_module(f".{_LAZY[name]}", __name__), name)
        globals()[name] = value
        return value
    raise AttributeError(f"module 'sdcguard_b200' has no attribute {name!r}")
