"""``python -m dsv41_train.rl.evaluate``: runs ``tiny_dsv41_b200.rl.evaluate``."""

from tiny_dsv41_b200.rl.evaluate import *  # noqa: F401,F403
from tiny_dsv41_b200.rl.evaluate import main

if __name__ == "__main__":
    main()
