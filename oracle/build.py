"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``needle_oracle.cpp`` — the C++ restatement of needle-rs's packed
CPU path — into ``oracle/liboracle.so``. Float contraction is off so every
fused multiply-add is the explicit ``fmaf`` (or vector fma, one rounding a
lane) the reference's ``mul_add`` calls for; ``-mfma -mavx2`` let those
compile to the hardware instructions and enable the vector integer sums.
"""

import os
import platform
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "needle_oracle.cpp")
LIB = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    # -O3 unrolls the fixed-length loops over vector accumulators (kept in
    # registers, not on the stack); it reassociates no float arithmetic
    flags = ["-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", "-ffp-contract=off", "-fno-fast-math"]
    if platform.machine() in ("x86_64", "AMD64"):
        flags += ["-mfma", "-mavx2"]
    tmp = LIB + ".tmp"
    subprocess.check_call(["g++", *flags, SRC, "-o", tmp])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
