"""Per-rank training worker (``python -m graspo_b200.cli.train_worker --config X``)."""

from __future__ import annotations

import argparse

from graspo_b200.core.schema import GraspoConfig


def main() -> None:
    parser = argparse.ArgumentParser(prog="python -m graspo_b200.cli.train_worker",
                                     description=("Per-rank process started by `graspo launch` (directly or through torchrun); "
                                                  "not meant to be run by hand."))
    parser.add_argument("--config", "-c", required=True)
    args = parser.parse_args()
    config = GraspoConfig.from_yaml(args.config)
    from graspo_b200.engine.runtime import GraspoFlowRuntime

    runtime = GraspoFlowRuntime.from_config(config)
    if config.train_method == "sft":
        from graspo_b200.train.sft_trainer import SFTTrainer

        SFTTrainer(config, runtime).train()
    else:
        from graspo_b200.cli.app import select_backend
        from graspo_b200.train.trainer import GraspoTrainer

        GraspoTrainer(config, runtime, selection=select_backend(config)).train()


if __name__ == "__main__":
    main()
