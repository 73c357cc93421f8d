"""``python train.py DATA --arch yoco_3b ...`` (run under torchrun for several GPUs); see faster_yoco_b200/cli/train.py."""
from faster_yoco_b200.cli.train import cli_main

if __name__ == "__main__":
    cli_main()
