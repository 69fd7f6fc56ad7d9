"""Build recipe for the in-tree drop-in library ``libgroupconv.so``.

One nvcc invocation compiles the C ABI (``csrc/common.cpp``) and the sm_100a
CUDA engine (``csrc/conv_cuda.cu``) into a shared library that sits next to
this file.  The CUDA runtime is linked as a shared library so that, inside a
process that already loaded PyTorch's CUDA runtime, both use one runtime
instance (one current device per thread, one primary context).

    python -m groupconv_atlas_b200.build          # build if stale
    python -m groupconv_atlas_b200.build --force  # always rebuild
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / 'csrc'
INCLUDE = ROOT / 'include'
LIBRARY = PACKAGE / 'libgroupconv.so'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def nvcc() -> str:
    for candidate in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc', shutil.which('nvcc')):
        if candidate and Path(candidate).exists():
            return candidate
    raise FileNotFoundError('nvcc not found: the B200 library needs the CUDA 12.9 toolkit')


def sources() -> list[Path]:
    return sorted(CSRC.glob('*.cu')) + sorted(CSRC.glob('*.cpp'))


def dependencies() -> list[Path]:
    return sources() + sorted(CSRC.glob('*.cuh')) + sorted(CSRC.glob('*.h')) + [INCLUDE / 'groupconv.h', Path(__file__)]


def stale(target: Path = LIBRARY) -> bool:
    if not target.exists():
        return True
    built = target.stat().st_mtime
    return any(p.stat().st_mtime > built for p in dependencies())


def command(output: Path = LIBRARY, extra: list[str] | None = None) -> list[str]:
    cuda_lib = Path(nvcc()).resolve().parent.parent / 'lib64'
    return [nvcc(), *ARCH, '-O3', '-lineinfo', '-std=c++17', '-shared',
            '-Xcompiler', '-fPIC,-Wall', '-Xptxas', '-warn-spills',
            '-cudart', 'shared', f'-I{INCLUDE}', f'-I{CSRC}',
            f'-Xlinker', f'-rpath,{cuda_lib}',
            *(extra or []), '-o', str(output), *map(str, sources())]


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile the library when a source is newer than it (or when forced)."""
    if not force and not stale():
        return LIBRARY
    tmp = LIBRARY.with_suffix('.so.part')
    cmd = command(tmp, extra)
    if verbose:
        print(' '.join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f'nvcc failed with exit code {result.returncode}')
    if verbose and (result.stdout or result.stderr):
        sys.stderr.write(result.stdout + result.stderr)
    tmp.replace(LIBRARY)
    return LIBRARY


TORCH_EXT_SOURCE = PACKAGE / 'torch_ext' / 'conv_op.cpp'


def torch_ext_path() -> Path:
    """The PyTorch binding's extension module next to this file."""
    import sysconfig
    return PACKAGE / ('_gcb_torch' + sysconfig.get_config_var('EXT_SUFFIX'))


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile the PyTorch front end (torch_ext/conv_op.cpp, a thin C++ caller
    of gc_cuda_conv that allocates the output with PyTorch) against the
    in-tree library, when it is older than its sources."""
    import sysconfig
    import torch
    from torch.utils import cpp_extension
    target = torch_ext_path()
    deps = [TORCH_EXT_SOURCE, INCLUDE / 'groupconv.h', LIBRARY, Path(__file__)]
    if not force and target.exists() and all(d.stat().st_mtime <= target.stat().st_mtime for d in deps):
        return target
    cuda_include = Path(nvcc()).resolve().parent.parent / 'include'
    torch_lib = cpp_extension.library_paths()[0]
    abi = int(torch.compiled_with_cxx11_abi())
    cmd = ['g++', '-O2', '-std=c++17', '-shared', '-fPIC', f'-D_GLIBCXX_USE_CXX11_ABI={abi}',
           '-DTORCH_EXTENSION_NAME=_gcb_torch', '-DTORCH_API_INCLUDE_EXTENSION_H',
           *[f'-I{d}' for d in cpp_extension.include_paths()], f'-I{sysconfig.get_paths()["include"]}',
           f'-I{cuda_include}', f'-I{INCLUDE}', str(TORCH_EXT_SOURCE),
           f'-L{PACKAGE}', '-lgroupconv', f'-L{torch_lib}', '-lc10', '-lc10_cuda', '-ltorch', '-ltorch_cpu',
           '-ltorch_python', f'-Wl,-rpath,$ORIGIN', f'-Wl,-rpath,{torch_lib}', '-o', str(target) + '.part']
    if verbose:
        print(' '.join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f'g++ failed with exit code {result.returncode}')
    Path(str(target) + '.part').replace(target)
    return target


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--force', action='store_true')
    parser.add_argument('--verbose', action='store_true')
    parser.add_argument('--ptxas-info', action='store_true', help='print registers/spills per kernel')
    args = parser.parse_args(argv)
    extra = ['-Xptxas', '-v'] if args.ptxas_info else None
    path = build(force=args.force or args.ptxas_info, verbose=args.verbose or args.ptxas_info, extra=extra)
    print(path)
    return 0


if __name__ == '__main__':
    raise SystemExit(main())
