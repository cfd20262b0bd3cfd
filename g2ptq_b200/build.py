"""Build libg2ptq_b200.so in-tree for sm_100a (``python -m g2ptq_b200.build``)."""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs=None, verbose=False):
    jobs = jobs or max(1, min(16, os.cpu_count() or 1))
    cmd = ["make", "-C", os.path.join(HERE, "csrc"), f"-j{jobs}"]
    res = subprocess.run(cmd, stdout=None if verbose else subprocess.PIPE,
                         stderr=subprocess.STDOUT, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout or "")
        raise RuntimeError("building libg2ptq_b200.so failed")
    return os.path.join(HERE, "_lib", "libg2ptq_b200.so")


if __name__ == "__main__":
    print(build(verbose=True))
