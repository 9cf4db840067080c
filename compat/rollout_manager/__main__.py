"""``python -m rollout_manager``: this library's rollout CLI."""

from tiny_dsv41_b200.rollout.cli import main

if __name__ == "__main__":
    main()
