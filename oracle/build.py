"""Builds the C oracle, oracle/liboracle.so -- TEST INFRASTRUCTURE ONLY (the CPU baseline and a cross-check of
the numpy oracle). The reference itself (strata-mlx) has no C/C++ sources to compile: its kernels are Metal
source in Python strings, so there is no oracle/_ref build.

    python oracle/build.py
"""

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "liboracle.so")


def build() -> str:
    import importlib.util

    spec = importlib.util.spec_from_file_location("oracle_gen_tables", os.path.join(HERE, "gen_tables.py"))
    gen_tables = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen_tables)

    hdr = os.path.join(HERE, "iq_tables_ref.h")
    text = gen_tables.render()
    if not os.path.exists(hdr) or open(hdr).read() != text:
        open(hdr, "w").write(text)
    src = os.path.join(HERE, "blocks_ref.c")
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(src), os.path.getmtime(hdr)):
        return OUT
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-std=c11",
           src, "-o", OUT, "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build())
