"""``dsv41_train.rl`` command-line modules (``train``, ``distributed_grpo``, ``sample``,
``evaluate``) backed by ``tiny_dsv41_b200.rl``; library modules resolve through the parent
package's import hook."""
