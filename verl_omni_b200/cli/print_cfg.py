"""Print the composed, resolved config: ``python -m verl_omni_b200.cli.print_cfg [name] [key=value ...]``."""

from __future__ import annotations

import sys

import yaml

from verl_omni_b200.utils.config import CONFIG_ROOT, load_config


def main(argv=None) -> None:
    argv = list(sys.argv[1:] if argv is None else argv)
    name = "diffusion_trainer"
    if argv and "=" not in argv[0] and (CONFIG_ROOT / f"{argv[0]}.yaml").exists():
        name = argv.pop(0)
    print(yaml.safe_dump(load_config(name, argv).to_dict(), sort_keys=False))


if __name__ == "__main__":
    main()
