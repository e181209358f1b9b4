"""Build the in-tree native libraries: inferenz_b200/libinzg.so (CUDA kernels for sm_100a + C ABI + host tools)."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs=8, verbose=False):
    cmd = ["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")]
    subprocess.run(cmd, check=True, stdout=None if verbose else subprocess.DEVNULL)
    return os.path.join(HERE, "libinzg.so")


if __name__ == "__main__":
    print(build(verbose=True))
