"""``python -m dsv41_train.rl.sample``: runs ``tiny_dsv41_b200.rl.sample``."""

from tiny_dsv41_b200.rl.sample import *  # noqa: F401,F403
from tiny_dsv41_b200.rl.sample import main

if __name__ == "__main__":
    main()
