"""``python -m dsv41_train.rl.distributed_grpo``: runs ``tiny_dsv41_b200.rl.distributed_grpo``."""

from tiny_dsv41_b200.rl.distributed_grpo import *  # noqa: F401,F403
from tiny_dsv41_b200.rl.distributed_grpo import main

if __name__ == "__main__":
    main()
