"""Typed run configuration: profiles, YAML overlays, CLI overrides and validation."""
import pytest

from qwen38_b200.runconfig import load_profiles, load_run_config, parse_override


def test_defaults_and_every_profile_validate():
    assert load_run_config().spec.block_rows == 16
    for name in load_profiles():
        cfg = load_run_config(profile=name)
        assert cfg.validate() is cfg


def test_overlay_order(tmp_path):
    p = tmp_path / "c.yaml"
    p.write_text("spec: {block_rows: 8}\nserving: {slots: 2}\n")
    cfg = load_run_config(str(p), profile="multi-stream-8x4k", overrides=["serving.slots=3", "kernels.pdl=true"])
    assert cfg.spec.block_rows == 8          # file over profile
    assert cfg.serving.slots == 3            # override over file
    assert cfg.serving.output_budget_multiple == 256   # from the profile
    assert cfg.kernels.pdl is True
    assert parse_override("runtime.max_context=4096") == {"runtime": {"max_context": "4096"}}
    assert load_run_config(overrides=["runtime.max_context=4096"]).runtime.max_context == 4096


@pytest.mark.parametrize("bad", [
    ["parallel.tp=3"], ["parallel.comm=gloo"], ["spec.block_rows=12"], ["kernels.ops=torch", "parallel.tp=2"],
    ["spec.drafter=mtp"], ["spec.drafter=lookup"], ["runtime.kv_block_size=8"], ["nosuch.field=1"],
    ["spec.nosuch=1"], ["kernels.pdl=maybe"],
])
def test_invalid_combinations_raise(bad):
    with pytest.raises(ValueError):
        load_run_config(overrides=bad)
