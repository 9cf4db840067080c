"""Build the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``.

The extension is compiled for Blackwell B200 only (``compute_100a`` / ``sm_100a``);
there is no other architecture and no JIT fallback.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(
    glob.glob(os.path.join("csrc", "*.cpp"))
)

NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("TDSV_PTXAS_VERBOSE") else "-O3",
    "-DNDEBUG",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
# Link the shared libstdc++ (the one torch uses): the toolchain wrapper's own search path only
# offers a dangling libstdc++.so symlink and would otherwise fall back to the static archive,
# giving the extension a private iostream/locale copy.
LINK_ARGS = []
for candidate in ("/usr/lib/gcc/x86_64-linux-gnu/13", "/usr/lib/gcc/x86_64-linux-gnu/12"):
    if os.path.exists(os.path.join(candidate, "libstdc++.so")):
        LINK_ARGS.append("-L" + candidate)
        break

if os.environ.get("TDSV_BOUNDS_CHECK"):
    NVCC_FLAGS.append("-DTDSV_BOUNDS_CHECK=1")

setup(
    name="tiny_dsv41_b200",
    version="0.1.0",
    packages=["tiny_dsv41_b200", "tiny_dsv41_b200.models", "tiny_dsv41_b200.models.dsv4",
              "tiny_dsv41_b200.models.qwen", "tiny_dsv41_b200.ops", "tiny_dsv41_b200.optim",
              "tiny_dsv41_b200.parallel", "tiny_dsv41_b200.rl", "tiny_dsv41_b200.rollout", "tiny_dsv41_b200.train",
              "tiny_dsv41_b200.utils",
              # drop-in module paths of the original packages (compat/): dsv41_train.*, rollout_manager.*
              "dsv41_train", "dsv41_train.rl", "rollout_manager"],
    package_dir={"dsv41_train": "compat/dsv41_train", "dsv41_train.rl": "compat/dsv41_train/rl",
                 "rollout_manager": "compat/rollout_manager"},
    package_data={"tiny_dsv41_b200.models.dsv4": ["tiny_config.json"]},
    entry_points={"console_scripts": [
        "rollout-manager = tiny_dsv41_b200.rollout.cli:main",
        "tdsv-rl-train = tiny_dsv41_b200.rl.train:main",
        "tdsv-sft = tiny_dsv41_b200.train.sft:main",
    ]},
    ext_modules=[
        CUDAExtension(
            name="tiny_dsv41_b200._C",
            sources=SOURCES,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            extra_link_args=LINK_ARGS,
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
