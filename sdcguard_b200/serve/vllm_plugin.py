"""vLLM plugin: vLLM's unquantized bf16 linear layers run on this package's checked tcgen05 GEMM while vLLM serves.

    SDCGUARD_B200=1 vllm serve <model>            # with this package installed (entry point vllm.general_plugins)
    # or in-process: sdcguard_b200.serve.vllm_plugin.register() before constructing vllm.LLM

Off unless SDCGUARD_B200=1 (vLLM loads every installed plugin). In each vLLM process that loads models:

  - after vLLM has loaded a linear layer's weights (`UnquantizedLinearMethod.process_weights_after_loading`), a
    bf16 layer on a CUDA device with both dimensions multiples of 8, selected by SDCGUARD_SHARE / SDCGUARD_OFFSET
    (the rule of `serve.settings`), gets its checksum rows built once and a row in the device's check state table;
  - its matmul (`UnquantizedLinearMethod.apply`) then runs as one custom operator, `sdcguard_b200_vllm::linear`,
    whose CUDA implementation is the checked GEMM: the layer's output is the checked kernel's own, and its check
    runs in the kernel's epilogue. The operator has a fake implementation, so vLLM's torch.compile keeps one graph
    and its CUDA graphs capture the kernel; the GEMM workspace is sized before capture for every batch size up to
    the scheduler's largest (max_num_batched_tokens);
  - every SDCGUARD_POLL_EVERY model steps (default 16) the state table is read without stalling the GPU (the read
    reports the previous one, as `ServeGuard.poll(wait=False)`), and after a step that ends SDCGUARD_POLL_SECONDS
    (default 2) or more after the last read it is read at once, waiting for the GPU; alarms are logged as
    `sdcguard ALERT` lines and appended to SDCGUARD_LOG as JSON events;
  - `coverage()` gives the layers checked and left out, with the reason, and the share of linear-layer weights
    checked. Layers left out (other dtypes, quantized methods, the LM head, outside the share) run vLLM's own GEMM;
  - with SDCGUARD_METRICS_PORT, each worker publishes the protection metrics of `serve.metrics` on that port plus
    its local rank (GET /metrics), so `sdcguard ready`, `decide` and `qualify` judge a running `vllm serve`; its token
    counter counts the tokens the worker computed;
  - with SDCGUARD_REQUIRE (1: every layer the share selects; a fraction such as 0.9: that share of them), the first
    model step refuses to serve (RuntimeError) when fewer are checked, or when none is;
  - with SDCGUARD_QUANT=1, weight-only INT4 / INT8 layers served by vLLM's mixed-precision kernels (Marlin, Machete
    and the others behind `MPLinearKernel`) are checked too: their effective bf16 weights are read before the kernel
    repacks them (`ops.quant.from_vllm`), the kernel itself is probed on unit vectors after the repack and must give
    those weights bit for bit (for Machete with zero points, whichever of its two roundings matches), and the layer
    then runs on the checked GEMM over the effective weights (kept in bf16: checked, not memory-saving). A layer the
    reader refuses or the probe contradicts stays on vLLM's kernel, with the reason in `coverage()`.

The reference's plugin (SDCGUARD=1) keeps vLLM's GEMM and adds a Triton check after it; here the check is part of
the GEMM, so a checked layer is still one launch. Differences in rounding order from cuBLAS's GEMM are in the last
bit of the bf16 outputs.

Reference: src/sdcguard/vllm_plugin.py:1-80 (what the plugin checks and its settings), `register` :2239, the
model-runner hook :2430-2501 (here the GPU worker's step, which both of vLLM 0.22's model runners serve).
"""
from __future__ import annotations

import logging
import os
import threading
import time
from typing import Optional

import torch

log = logging.getLogger("sdcguard_b200")

ENV = "SDCGUARD_B200"
_STATE: dict = {}          # device -> DeviceState
_LAYERS: list = []         # layer id -> (name, CheckedWeight, slot, device)
_LEFT_OUT: list = []       # (name, reason, weight elements)
_COUNTERS = {"polls": 0, "requests": 0, "prompt_tokens": 0, "generated_tokens": 0, "longest_prompt": 0, "steps": 0,
             "tokens_computed": 0}
_EXPORTER: list = []
_STARTED = [0.0]
_LOCK = threading.Lock()
_REGISTERED = [False]
_COUNTER = [0]             # linear layers seen (selection index)
_LIB = None


class DeviceState:
    def __init__(self, device: torch.device):
        from ..ops import gemm
        from .settings import CheckSettings
        self.device = device
        self.settings = CheckSettings.from_env()
        self.state = gemm.StateTable(device, 512)
        self.slot_weights: dict = {}
        self.steps = 0
        self.guard = None
        self.last_read = 0.0          # time of the last read of the state table
        self.tokens_at_read = 0       # tokens computed when the read in flight was started
        gemm.enable_capture(device)
        _start_exporter(device)


def _max_tokens() -> int:
    try:
        from vllm.config import get_current_vllm_config_or_none
        cfg = get_current_vllm_config_or_none()
        if cfg is not None and cfg.scheduler_config is not None:
            return int(cfg.scheduler_config.max_num_batched_tokens)
    except Exception:  # noqa: BLE001  (older vLLM: use the setting)
        pass
    return int(os.environ.get("SDCGUARD_B200_MAX_TOKENS", "16384"))


def _state(device: torch.device) -> DeviceState:
    st = _STATE.get(device)
    if st is None:
        from ..ops import verify
        verify.verified(device)               # the kernels reproduce their references on this device first
        st = _STATE[device] = DeviceState(device)
    return st


def _layer_name(layer: torch.nn.Module) -> str:
    return getattr(layer, "prefix", None) or f"linear{_COUNTER[0]}"


def _adopt(layer: torch.nn.Module, weight: Optional[torch.Tensor] = None, label: str = "ABFT GEMM") -> None:
    """Checksums of a loaded linear layer and its state row, when it can be checked (`weight`: the matrix the
    layer multiplies by, when it is not the layer's own `weight`)."""
    from ..ops import gemm
    from .settings import layer_selected
    w = weight if weight is not None else getattr(layer, "weight", None)
    name = _layer_name(layer)
    lid = getattr(layer, "_sdcguard_b200_id", None)
    if lid is not None:                 # weights loaded again: new checksums, same state row
        name0, _, slot, dev, add_bias = _LAYERS[lid]
        bias = getattr(layer, "bias", None) if add_bias else None
        cw = gemm.CheckedWeight(w.detach(), None if bias is None else bias.detach())
        _STATE[dev].slot_weights[slot] = cw
        _LAYERS[lid] = (name0, cw, slot, dev, add_bias)
        return
    with _LOCK:
        i = _COUNTER[0]
        _COUNTER[0] += 1
    why = None
    if w is None or not isinstance(w, torch.Tensor):
        why = "no weight tensor"
    elif w.device.type != "cuda":
        why = "not on a CUDA device"
    elif w.dtype != torch.bfloat16 or w.dim() != 2:
        why = f"weight {w.dtype} {tuple(w.shape)} (the checked GEMM multiplies 2-D bf16)"
    elif w.shape[0] % 8 or w.shape[1] % 8:
        why = f"shape {tuple(w.shape)}: n and k must be multiples of 8"
    if why is None:
        st = _state(w.device)
        if not layer_selected(i, st.settings.share, st.settings.offset):
            why = f"outside the share {st.settings.share:g}"
    if why is not None:
        _LEFT_OUT.append((name, why, int(w.numel()) if isinstance(w, torch.Tensor) else 0))
        return
    bias = getattr(layer, "bias", None) if weight is None else None     # (quantized kernels get it in apply)
    add_bias = bias is not None and not getattr(layer, "skip_bias_add", False)
    cw = gemm.CheckedWeight(w.detach(), bias.detach() if add_bias else None)
    slot = st.state.add(f"{name} ({label})", cw.nb)
    st.slot_weights[slot] = cw
    # the workspace is sized now, before vLLM captures CUDA graphs, for every batch size the scheduler can form
    gemm.reserve_for_rows(w.device, cw.n, _max_tokens())
    gemm.error_word(w.device)
    with _LOCK:
        layer._sdcguard_b200_id = len(_LAYERS)
        _LAYERS.append((name, cw, slot, w.device, add_bias))


def _linear_impl(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], layer: int) -> torch.Tensor:
    from ..ops import gemm
    name, cw, slot, dev, add_bias = _LAYERS[layer]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    st = _STATE[dev]
    y = gemm.checked_linear(x2, cw, st.state.state, slot, z_alarm=st.settings.z_alarm)
    if bias is not None and not add_bias:
        y = y + bias
    return y.view(*x.shape[:-1], cw.n)


def _linear_fake(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], layer: int) -> torch.Tensor:
    return x.new_empty(*x.shape[:-1], weight.shape[0])


def _define_op() -> None:
    global _LIB
    if _LIB is not None:
        return
    _LIB = torch.library.Library("sdcguard_b200_vllm", "DEF")
    _LIB.define("linear(Tensor x, Tensor weight, Tensor? bias, int layer) -> Tensor")
    _LIB.impl("linear", _linear_impl, "CUDA")
    _LIB._register_fake("linear", _linear_fake)


def _poll(dev: torch.device, wait: bool = False) -> list:
    """Read the device's check state (non-blocking unless wait) and log alarms."""
    st = _STATE[dev]
    if st.guard is None:
        from ..utils.events import EventLog
        from .guard import ServeGuard
        st.guard = ServeGuard(st, z_alarm=st.settings.z_alarm, log=EventLog(os.environ.get("SDCGUARD_LOG")))
    events = st.guard.poll(wait=wait)
    for ev in events:
        log.error("sdcguard ALERT: %s on %s: %s", ev.detail.get("layer"), dev, {k: v for k, v in ev.detail.items()
                                                                                  if k != "layer"})
    return events


def require_ok(checked: int, left_out: list, value: Optional[str]) -> Optional[str]:
    """Why SDCGUARD_REQUIRE refuses (None: it does not). Layers left out by the share count as not selected."""
    if not value:
        return None
    try:
        need = float(value)
    except ValueError:
        return f"SDCGUARD_REQUIRE={value!r} is not 1 or a fraction"
    selected_out = [r for r in left_out if not r[1].startswith("outside the share")]
    total = checked + len(selected_out)
    if checked == 0:
        return "no linear layer is checked"
    share = checked / total
    if share + 1e-12 < min(1.0, need):
        reasons: dict = {}
        for r in selected_out:
            reasons[r[1].split(":")[0]] = reasons.get(r[1].split(":")[0], 0) + 1
        return (f"{checked} of {total} selected linear layers are checked ({share:.1%}), SDCGUARD_REQUIRE={value}; "
                f"left out: {reasons}")
    return None


def _after_step(scheduler_output=None) -> None:
    every = max(1, int(os.environ.get("SDCGUARD_POLL_EVERY", "16")))
    _COUNTERS["steps"] += 1
    if _COUNTERS["steps"] == 1:
        why = require_ok(len(_LAYERS), _LEFT_OUT, os.environ.get("SDCGUARD_REQUIRE"))
        if why is not None:
            raise RuntimeError(f"sdcguard_b200: refusing to serve: {why}")
    if scheduler_output is not None:
        n = getattr(scheduler_output, "total_num_scheduled_tokens", 0) or 0
        per = getattr(scheduler_output, "num_scheduled_tokens", None) or {}
        _COUNTERS["tokens_computed"] += int(n)
        _COUNTERS["requests"] += len(per)
        if per:
            _COUNTERS["longest_prompt"] = max(_COUNTERS["longest_prompt"], max(int(v) for v in per.values()))
    poll_seconds = float(os.environ.get("SDCGUARD_POLL_SECONDS", "2"))
    now = time.time()
    for dev, st in list(_STATE.items()):
        st.steps += 1
        late = now - st.last_read >= poll_seconds
        if st.steps % every == 0 or late:
            # a step long after the last read: read now, waiting for the GPU once, so a lightly loaded server reports
            # within a step; otherwise the read reports the one started at the previous poll
            _poll(dev, wait=late)
            _COUNTERS["polls"] += 1
            # the published token counter covers what the folded read covers, so checks and tokens move together
            _COUNTERS["generated_tokens"] = _COUNTERS["tokens_computed"] if late else st.tokens_at_read
            st.tokens_at_read = _COUNTERS["tokens_computed"]
            st.last_read = now


def _check_coverage() -> dict:
    checked = sum(cw.n * cw.k for _, cw, _, _, _ in _LAYERS)
    left = sum(r[2] for r in _LEFT_OUT)
    return {"layers_checked": len(_LAYERS), "layers_unchecked": len(_LEFT_OUT), "fp8_layers_checked": 0,
            "weights_checked_ratio": checked / (checked + left) if checked + left else 0.0}


def metrics_text(dev: torch.device) -> str:
    """The protection metrics of this worker (the device's state as of its last poll)."""
    from .. import __version__
    from .metrics import render, settings_labels
    st = _STATE.get(dev)
    cov = st.guard.coverage_report() if st is not None and st.guard is not None else {}
    props = torch.cuda.get_device_properties(dev) if dev.type == "cuda" else None
    worker = {"gpu": props.name if props else "cpu", "uuid": str(getattr(props, "uuid", "")) if props else "",
              "pid": os.getpid(), "started": int(_STARTED[0]), "device": dev}
    model = ""
    try:
        from vllm.config import get_current_vllm_config_or_none
        cfg = get_current_vllm_config_or_none()
        model = cfg.model_config.model if cfg is not None and cfg.model_config is not None else ""
    except Exception:  # noqa: BLE001  (no vLLM config readable: the model name stays empty)
        pass
    try:
        import vllm
        vllm_version = vllm.__version__
    except Exception:  # noqa: BLE001
        vllm_version = ""
    stack = {"model": model, "precision": "bf16", "checked": "true", "torch": torch.__version__,
             "cuda": torch.version.cuda, "weights_digest": "", "version": __version__, "engine": f"vllm {vllm_version}"}
    settings = st.settings if st is not None else None
    z = settings.z_alarm if settings is not None else 6.0
    counters = dict(_COUNTERS, polls=_COUNTERS["polls"])
    return render(cov, _check_coverage(), counters, worker, stack, settings_labels(settings, z, False), z)


def _start_exporter(dev: torch.device) -> None:
    port = os.environ.get("SDCGUARD_METRICS_PORT")
    if not port or _EXPORTER:
        return
    import time as _time
    from .metrics import Exporter
    _STARTED[0] = _time.time()
    rank = int(os.environ.get("LOCAL_RANK", dev.index if dev.index is not None else 0))
    _EXPORTER.append(Exporter(int(port) + rank, lambda: metrics_text(dev)))
    log.info("sdcguard_b200: protection metrics on port %d", int(port) + rank)


def coverage() -> dict:
    """Layers checked, layers left out (with reasons), the share of linear-layer weight elements checked, and the
    serving guard's counts per device (after a final blocking read)."""
    checked_el = sum(cw.n * cw.k for _, cw, _, _, _ in _LAYERS)
    out = {"layers_checked": len(_LAYERS), "layers_left_out": len(_LEFT_OUT),
           "left_out": [(n, r) for n, r, _ in _LEFT_OUT[:64]], "checked_weight_elements": checked_el,
           "weights_checked_ratio": _check_coverage()["weights_checked_ratio"], "devices": {}}
    for dev, st in _STATE.items():
        _poll(dev, wait=True)
        _COUNTERS["generated_tokens"] = _COUNTERS["tokens_computed"]
        st.tokens_at_read, st.last_read = _COUNTERS["tokens_computed"], time.time()
        out["devices"][str(dev)] = st.guard.coverage_report()
    return out


def _patch() -> None:
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod
    orig_load = UnquantizedLinearMethod.process_weights_after_loading
    orig_apply = UnquantizedLinearMethod.apply

    def process_weights_after_loading(self, layer):
        orig_load(self, layer)
        try:
            _adopt(layer)
        except Exception as e:  # noqa: BLE001  (a layer that cannot be adopted runs vLLM's GEMM, counted)
            w = getattr(layer, "weight", None)
            _LEFT_OUT.append((_layer_name(layer), f"not adopted: {type(e).__name__}: {e}"[:200],
                              int(w.numel()) if isinstance(w, torch.Tensor) else 0))

    def apply(self, layer, x, bias=None):
        lid = getattr(layer, "_sdcguard_b200_id", None)
        if lid is None or x.dtype != torch.bfloat16:
            return orig_apply(self, layer, x, bias)
        return torch.ops.sdcguard_b200_vllm.linear(x, layer.weight, bias, lid)

    UnquantizedLinearMethod.process_weights_after_loading = process_weights_after_loading
    UnquantizedLinearMethod.apply = apply
    # the GPU worker's step (whichever model runner, V1 or V2, it was built with) gets the scheduler's output
    try:
        from vllm.v1.worker.gpu_worker import Worker
    except ImportError:
        log.warning("sdcguard_b200: no vLLM GPU worker to hook; results are read only by coverage()")
        return
    orig_exec = Worker.execute_model

    def execute_model(self, *a, **kw):
        out = orig_exec(self, *a, **kw)
        _after_step(a[0] if a else kw.get("scheduler_output"))
        return out

    Worker.execute_model = execute_model


def _quant_kernel_classes() -> list:
    """vLLM's concrete mixed-precision linear kernel classes (every imported subclass of MPLinearKernel)."""
    import importlib
    import pkgutil
    from vllm.model_executor.kernels.linear import mixed_precision as mp
    from vllm.model_executor.kernels.linear.mixed_precision.MPLinearKernel import MPLinearKernel
    for m in pkgutil.iter_modules(mp.__path__):
        try:
            importlib.import_module(f"{mp.__name__}.{m.name}")
        except Exception:  # noqa: BLE001  (a backend module that cannot import here has no layers here)
            pass
    out, todo = [], list(MPLinearKernel.__subclasses__())
    while todo:
        c = todo.pop()
        out.append(c)
        todo += c.__subclasses__()
    return out


def _adopt_quant(layer, kernel, qw, orig_apply) -> None:
    """After the kernel's repack: probe it against the effective weights read before, then adopt the layer."""
    from ..ops import quant
    w = qw.effective_weight()
    cols = quant.probe_columns(qw.k, qw.group, limit=int(os.environ.get("SDCGUARD_QUANT_PROBE_COLUMNS", "256")))
    tried = []
    for cand in ([qw] + ([qw.with_zero_mode(m) for m in quant.ZERO_MODES if m != qw.zero_mode]
                         if qw.zeros is not None else [])):
        w = cand.effective_weight() if cand is not qw else w
        r = quant.probe(lambda x: orig_apply(kernel, layer, x, None), w, cols)
        tried.append(f"{cand.zero_mode}: {r['mismatches']} of {r['columns'] * w.shape[0]}")
        if r["ok"]:
            layer._sdcguard_b200_weff = w
            _adopt(layer, weight=w, label=f"ABFT GEMM, INT{qw.bits} effective weights ({cand.zero_mode})")
            return
    _LEFT_OUT.append((_layer_name(layer), "quantized kernel differs from the restated weights (" +
                      "; ".join(tried) + ")", qw.n * qw.k))


def _patch_quant(classes=None) -> list:
    """SDCGUARD_QUANT=1: the mixed-precision kernels' weight loading and apply (see the module docstring)."""
    from ..ops import quant
    patched = []
    for cls in (classes if classes is not None else _quant_kernel_classes()):
        if "process_weights_after_loading" not in cls.__dict__ or "apply_weights" not in cls.__dict__:
            continue
        orig_load, orig_apply = cls.__dict__["process_weights_after_loading"], cls.__dict__["apply_weights"]

        def process_weights_after_loading(self, layer, _load=orig_load, _apply=orig_apply):
            qw, why = None, None
            try:
                qw = quant.from_vllm(layer, self)
            except Exception as e:  # noqa: BLE001  (the reason is recorded; vLLM's own path is untouched)
                why = f"quantized layer not read: {type(e).__name__}: {e}"[:200]
            _load(self, layer)
            if qw is None:
                shape = getattr(getattr(self, "config", None), "partition_weight_shape", (0, 0))
                _LEFT_OUT.append((_layer_name(layer), why, int(shape[0]) * int(shape[1])))
                return
            try:
                _adopt_quant(layer, self, qw, _apply)
            except Exception as e:  # noqa: BLE001
                _LEFT_OUT.append((_layer_name(layer), f"not adopted: {type(e).__name__}: {e}"[:200], qw.n * qw.k))

        def apply_weights(self, layer, x, bias=None, _apply=orig_apply):
            lid = getattr(layer, "_sdcguard_b200_id", None)
            if lid is None or x.dtype != torch.bfloat16:
                return _apply(self, layer, x, bias)
            return torch.ops.sdcguard_b200_vllm.linear(x, layer._sdcguard_b200_weff, bias, lid)

        cls.process_weights_after_loading = process_weights_after_loading
        cls.apply_weights = apply_weights
        patched.append(cls)
    return patched


def register() -> None:
    """vLLM general-plugin entry point (and the in-process hook): patch vLLM once, when SDCGUARD_B200=1."""
    if os.environ.get(ENV, "0") != "1" or _REGISTERED[0]:
        return
    _define_op()
    _patch()
    if os.environ.get("SDCGUARD_QUANT", "0") == "1":
        try:
            names = [c.__name__ for c in _patch_quant()]
            log.info("sdcguard_b200: quantized linear kernels checked: %s", ", ".join(names) or "none found")
        except ImportError as e:
            log.warning("sdcguard_b200: no vLLM mixed-precision kernels to hook (%s)", e)
    _REGISTERED[0] = True
    log.info("sdcguard_b200: vLLM linear layers will run on the checked GEMM")
