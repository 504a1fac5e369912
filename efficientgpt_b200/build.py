"""Build step for the CUDA library (in-tree, sm_100a only).

    python -m efficientgpt_b200.build          # -> efficientgpt_b200/_lib/libegpt_b200.so

The library is one nvcc translation unit (csrc/egpt_b200.cu) compiled for `sm_100a` with the static CUDA
runtime, so the .so only needs the driver at run time and travels with the source tree.
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / 'csrc'
LIB_DIR = PKG / '_lib'
LIB = LIB_DIR / 'libegpt_b200.so'
SOURCES = ['egpt_b200.cu', 'capi.cu', 'elementwise.cu', 'gemv_i8.cu', 'attention.cu', 'decode_step.cu', 'decode_dataflow.cu', 'gemv_tc.cu', 'sampling.cu', 'gemm_tc.cu', 'attn_prefill.cu', 'attn_stream.cu', 'common.cuh',
           'internal.h']
HEADER = PKG.parent / 'include' / 'egpt_b200.h'


def nvcc_path():
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError('nvcc not found: the CUDA library cannot be built')


def nvcc_flags(ptxas_verbose=False):
    flags = ['-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '-lineinfo', '-std=c++17', '--expt-relaxed-constexpr',
             '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden', '-cudart', 'static', '-shared']
    if ptxas_verbose:
        flags += ['-Xptxas', '-v']
    return flags


def up_to_date():
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + [HEADER]
    return all(d.stat().st_mtime <= t for d in deps if d.exists())


def build(force=False, ptxas_verbose=False, quiet=False):
    """Compile csrc/ into _lib/libegpt_b200.so (skipped when it is newer than every source)."""
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix('.so.tmp')
    cmd = [nvcc_path(), *nvcc_flags(ptxas_verbose), '-o', str(tmp), str(CSRC / 'egpt_b200.cu')]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError('nvcc failed:\n' + ' '.join(cmd) + '\n' + res.stdout + res.stderr)
    if not quiet and (ptxas_verbose or res.stderr.strip()):
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    out = build(force='--force' in sys.argv, ptxas_verbose='-v' in sys.argv)
    print(out)
