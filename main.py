"""``python main.py --config ...`` == ``nano-megatron-train --config ...``."""

from nano_megatron_b200.cli.train import main

if __name__ == "__main__":
    main()
