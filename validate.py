"""``python validate.py --task harness_eval ...``; see faster_yoco_b200/cli/validate.py."""
from faster_yoco_b200.cli.validate import cli_main

if __name__ == "__main__":
    cli_main()
