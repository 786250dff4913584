"""The committed flattened config snapshots (``trainer/config/_generated_*.yaml``) match the config tree."""

from verl_omni_b200.cli import gen_config


def test_generated_config_snapshots_are_current():
    assert gen_config.main(["--check"]) == 0, "run: python -m verl_omni_b200.cli.gen_config"
