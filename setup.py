"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``."""
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("autodrive_b200", "csrc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

ext = CUDAExtension(
    name="autodrive_b200._C",
    sources=[os.path.join(CSRC, f) for f in (
        "bindings.cpp", "adstar_cpu.cpp", "sim.cu", "policy_ops.cu", "policy_tc.cu", "tc_gemm.cu", "comm_ops.cu", "noalloc_adam.cu", "sha256.cu", "plan_a.cu", "layernorm.cu", "attention.cu")],
    include_dirs=[os.path.join(HERE, CSRC)],
    extra_compile_args={
        "cxx": ["-O3", "-std=c++17"],
        "nvcc": ARCH + ["-O3", "-lineinfo", "-std=c++17", "--use_fast_math",
                        "--expt-relaxed-constexpr",
                        "-Xptxas", "-v"] if os.environ.get("AD_PTXAS_VERBOSE") else
                ARCH + ["-O3", "-lineinfo", "-std=c++17", "--use_fast_math",
                        "--expt-relaxed-constexpr"],
    },
)

class BuildWithManifest(BuildExtension.with_options(use_ninja=True)):
    """Build, then record the in-tree binary's digest and its sources'
    digests in autodrive_b200/_C.manifest.json (checked at run time by
    ``autodrive_b200.ops.ext.native_extension_identity``)."""

    def run(self):
        super().run()
        import importlib.util
        spec = importlib.util.spec_from_file_location(
            "_ad_ext", os.path.join(HERE, "autodrive_b200", "ops", "ext.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        for e in self.extensions:
            built = os.path.join(HERE, *e.name.split(".")[:-1], os.path.basename(self.get_ext_filename(e.name)))
            if os.path.exists(built):
                mod.write_build_manifest(built)


setup(
    name="autodrive-b200",
    version="0.1.0",
    packages=find_packages(include=["autodrive_b200*", "frc_defense*"]),
    ext_modules=[ext],
    cmdclass={"build_ext": BuildWithManifest},
    entry_points={"console_scripts": [
        "frc-defense=frc_defense.tensor_training:main",
        "frc-defense-tensor=frc_defense.tensor_training:main",
        "frc-defense-dashboard=frc_defense.dashboard:main",
    ]},
)
