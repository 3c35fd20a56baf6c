"""Builds styx_b200/host/generate_moe.c (the C host of the decode step)
against include/ and the built libstyx_moe.so, for the tests."""
import os
import shutil
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "styx_b200", "host", "generate_moe.c")
LIBDIR = os.path.join(ROOT, "styx_b200")


def build(out_dir) -> str:
    cc = shutil.which("gcc") or shutil.which("cc")
    exe = os.path.join(str(out_dir), "generate_moe")
    subprocess.run([cc, "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), SRC,
                    "-L", LIBDIR, "-lstyx_moe", f"-Wl,-rpath,{LIBDIR}", "-o", exe], check=True)
    return exe
