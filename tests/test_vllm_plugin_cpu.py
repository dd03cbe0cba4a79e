"""The vLLM plugin's host side (no GPU): off without SDCGUARD_B200=1, patches vLLM's unquantized linear method once
when on, registers its custom operator with a fake implementation, leaves a layer it cannot check on vLLM's GEMM
with the reason, and the selection follows the share."""
import os

import pytest
import torch


@pytest.fixture(scope="module")
def plugin():
    pytest.importorskip("vllm")
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod
    from sdcguard_b200.serve import vllm_plugin
    before = (UnquantizedLinearMethod.apply, UnquantizedLinearMethod.process_weights_after_loading)
    old = os.environ.pop("SDCGUARD_B200", None)
    vllm_plugin.register()                     # off: nothing patched
    assert UnquantizedLinearMethod.apply is before[0]
    os.environ["SDCGUARD_B200"] = "1"
    vllm_plugin.register()
    vllm_plugin.register()                     # once only
    yield vllm_plugin, UnquantizedLinearMethod, before
    UnquantizedLinearMethod.apply, UnquantizedLinearMethod.process_weights_after_loading = before
    if old is None:
        os.environ.pop("SDCGUARD_B200", None)
    else:
        os.environ["SDCGUARD_B200"] = old


def test_patched_and_falls_back_on_cpu(plugin):
    vp, ULM, before = plugin
    assert ULM.apply is not before[0] and ULM.process_weights_after_loading is not before[1]
    from vllm.v1.worker.gpu_worker import Worker
    assert Worker.execute_model.__name__ == "execute_model" and Worker.execute_model.__module__.endswith("vllm_plugin")
    assert hasattr(torch.ops.sdcguard_b200_vllm, "linear")
    layer = torch.nn.Module()
    layer.weight = torch.nn.Parameter(torch.randn(64, 32, dtype=torch.bfloat16), requires_grad=False)
    layer.prefix = "model.layers.0.mlp.down_proj"
    m = ULM()
    m.process_weights_after_loading(layer)
    assert not hasattr(layer, "_sdcguard_b200_id")
    assert ("model.layers.0.mlp.down_proj", "not on a CUDA device", 64 * 32) in vp._LEFT_OUT
    x = torch.randn(5, 32, dtype=torch.bfloat16)
    torch.testing.assert_close(m.apply(layer, x), torch.nn.functional.linear(x, layer.weight))
    fake = vp._linear_fake(x, layer.weight, None, 0)
    assert fake.shape == (5, 64)
    cov = vp.coverage()
    assert cov["layers_checked"] == 0 and cov["layers_left_out"] >= 1


def test_require_and_metrics_exporter(plugin):
    """SDCGUARD_REQUIRE's rule, and the per-worker exporter serving the protection metrics `ready` reads."""
    vp, _, _ = plugin
    assert vp.require_ok(3, [], None) is None
    assert vp.require_ok(3, [("a", "outside the share 0.5", 10)], "1") is None      # not selected: fine
    assert "3 of 4" in vp.require_ok(3, [("a", "weight torch.float32 (2, 2)", 4)], "1")
    assert vp.require_ok(3, [("a", "weight x", 4)], "0.7") is None
    assert vp.require_ok(0, [], "0.1") == "no linear layer is checked"
    from sdcguard_b200.serve.metrics import Exporter
    from sdcguard_b200.tools import _client
    ex = Exporter(0, lambda: vp.metrics_text(torch.device("cpu")), host="127.0.0.1")
    try:
        m = _client.scrape(f"http://127.0.0.1:{ex.port}")
        assert m["sdcguard_protected"] == 1 and "sdcguard_layers_checked" in m and "sdcguard_alarm_line" in m
        info = m["sdcguard_stack_info{}"][0][0]
        assert info["engine"].startswith("vllm") and info["checked"] == "true"
        assert m["sdcguard_worker_info{}"][0][0]["gpu"] == "cpu"
    finally:
        ex.close()
