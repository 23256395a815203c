"""Build script of connex-b200.

Two native modules are built in-tree (``python setup.py build_ext --inplace``):

* ``connex_b200._C``        -- the sm_100a CUDA kernels (tcgen05 GEMM, attention,
                               fused KV push, EP dispatch/combine, weight sync)
                               and the CUDA IPC plumbing, bound with pybind11.
* ``connex_b200._cxengine`` -- the C++17 transfer engine (identity-keyed
                               endpoints, host and GPU regions, one-sided
                               read/write, put_chain, events, heartbeats, VMM
                               export and the dead-peer graveyard) that
                               provides the data-plane surface of the control
                               plane.

Every CUDA file is compiled for exactly one target: sm_100a (B200).
"""
import os
import glob

from setuptools import Extension, setup, find_packages
from torch.utils.cpp_extension import CUDA_HOME, BuildExtension, CUDAExtension, CppExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
KDIR = os.path.join("connex_b200", "csrc", "kernels")
EDIR = os.path.join("connex_b200", "csrc", "engine")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]

kernel_sources = sorted(glob.glob(os.path.join(KDIR, "*.cu")) + glob.glob(os.path.join(KDIR, "*.cpp")))
engine_sources = sorted(glob.glob(os.path.join(EDIR, "*.cpp")))

ext_modules = [
    CUDAExtension(
        name="connex_b200._C",
        sources=kernel_sources,
        include_dirs=[os.path.join(ROOT, KDIR)],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]
if engine_sources:
    # plain pybind11 module: importing the engine loads neither libtorch nor
    # libcuda (the driver API is resolved at run time; cuda.h gives the types)
    import pybind11
    ext_modules.append(
        Extension(
            name="connex_b200._cxengine",
            sources=engine_sources,
            include_dirs=[os.path.join(ROOT, EDIR), pybind11.get_include(),
                          os.path.join(CUDA_HOME or "/usr/local/cuda", "include")],
            extra_compile_args=CXX_FLAGS + ["-pthread", "-fvisibility=hidden"],
            extra_link_args=["-pthread", "-ldl"],
            language="c++",
        )
    )

setup(
    name="connex-b200",
    version="0.2.1",
    description="B200-native endpoint-mobility communication framework for dynamic LLM serving",
    packages=find_packages(include=["connex", "connex.*", "connex_b200", "connex_b200.*"]),
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    python_requires=">=3.10",
    entry_points={
        "console_scripts": [
            "connex-front-router=connex.front_router:main",
            "connex-directory=connex.directory_server:main",
            "connex-pd-router=connex.serving.pd_router:main",
            "connex-proxy=connex.serving.proxy:main",
        ],
        # upstream engines find the plugins by name (no fork)
        "vllm.general_plugins": [
            "connex_pd = connex.adapters.vllm.plugin:register",
            "connex_rl = connex.rl.vllm_plugin:register",
            "connex_ep = connex.ep.vllm_ext:register",
        ],
        "sglang.srt.plugins": [
            "connex = connex.adapters.sglang.pd_backend:register",
            "connex_ep = connex.ep.sglang_ext:register",
        ],
    },
)
