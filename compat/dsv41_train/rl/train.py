"""``python -m dsv41_train.rl.train``: runs ``tiny_dsv41_b200.rl.train``."""

from tiny_dsv41_b200.rl.train import *  # noqa: F401,F403
from tiny_dsv41_b200.rl.train import main

if __name__ == "__main__":
    main()
