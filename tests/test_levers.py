"""The lever registry (flyai_b200.levers): requested vs observed per lever, unknown
flags, strict mode -- host logic only, no GPU."""
import pytest

from flyai_b200 import deepseek, gpt_oss, levers, m25


@pytest.fixture(autouse=True)
def fresh(monkeypatch):
    monkeypatch.setattr(gpt_oss, "_ATTEMPTS", [0])
    monkeypatch.setattr(gpt_oss, "_INSTALLED", [])
    monkeypatch.setattr(deepseek, "_ATTEMPTS", [0])
    monkeypatch.setattr(deepseek, "_INSTALLED", [])
    monkeypatch.setattr(m25, "_ATTEMPTS", [0])
    monkeypatch.setattr(m25, "_INSTALLED", [])


def verdicts(env):
    return {r["env"]: r["verdict"] for r in levers.audit(env)}


def test_idle_process_has_no_findings():
    v = verdicts({})
    assert set(v.values()) == {"UNUSED"}
    assert levers.check({"FLYAI_MOE_LEVERS_STRICT": "1"})


def test_flag_on_but_nothing_installed_is_a_mismatch(monkeypatch):
    monkeypatch.setattr(gpt_oss, "ENABLED", True)
    assert verdicts({"FLYAI_MOE_B200": "1"})["FLYAI_MOE_B200"] == "MISMATCH"
    with pytest.raises(RuntimeError):
        levers.check({"FLYAI_MOE_B200": "1", "FLYAI_MOE_LEVERS_STRICT": "1"})


def test_flag_set_after_import_is_a_mismatch(monkeypatch):
    monkeypatch.setattr(m25, "ENABLED", True)
    assert verdicts({"FLYAI_MOE_M25": "0"})["FLYAI_MOE_M25"] == "MISMATCH"


def test_unknown_flag_is_reported():
    assert verdicts({"FLYAI_MOE_DEEPSEK": "1"})["FLYAI_MOE_DEEPSEK"] == "UNKNOWN"
    assert "FLYAI_MOE_CHECK" not in verdicts({"FLYAI_MOE_CHECK": "1"})


def test_installed_lever_with_its_flag_is_ok(monkeypatch):
    class Stage:
        def __init__(self):
            self.moe = object()
    monkeypatch.setattr(m25, "ENABLED", True)
    layers = [Stage(), Stage()]

    class Fake(m25.Nvfp4MoE):
        def __init__(self):
            pass
    assert m25.install(layers, lambda layer: Fake()) == 2
    assert all(isinstance(layer._flyai_prev_moe, object) for layer in layers)
    assert verdicts({"FLYAI_MOE_M25": "1"})["FLYAI_MOE_M25"] == "OK"
    layers[0].moe = layers[0]._flyai_prev_moe       # something put the old module back
    assert verdicts({})["FLYAI_MOE_M25"] == "OK"    # one layer still live
    layers[1].moe = layers[1]._flyai_prev_moe
    assert verdicts({})["FLYAI_MOE_M25"] == "MISMATCH"   # requested, nothing live
