"""Environment check for the B200 build.

Replaces ghostweight_triton/utils/compat.py:11-74, which checks for an sm_120
GPU and TORCH_CUDA_ARCH_LIST for Triton. Here the requirements are an sm_100
(B200) GPU and the in-tree native library; Triton is not used.
"""

from __future__ import annotations

import os


def check_environment(verbose: bool = True) -> dict:
    """Report torch / CUDA / GPU / native-library readiness.

    Returns a dict with the reference's keys (torch_version, triton_version,
    cuda_version, cuda_available, gpu_name, compute_cap, arch_list_set,
    sm120_ready, warnings) plus sm100_ready and native_library.
    """
    info: dict = {"warnings": []}
    try:
        import torch

        info["torch_version"] = torch.__version__
        info["cuda_available"] = torch.cuda.is_available()
        if info["cuda_available"]:
            info["gpu_name"] = torch.cuda.get_device_name(0)
            cc = torch.cuda.get_device_capability(0)
            info["compute_cap"] = f"{cc[0]}.{cc[1]}"
            info["cuda_version"] = torch.version.cuda or "unknown"
        else:
            info["gpu_name"] = "N/A"
            info["compute_cap"] = "N/A"
            info["cuda_version"] = "N/A"
            info["warnings"].append("CUDA not available - kernels will not run.")
    except ImportError:
        info["torch_version"] = "NOT INSTALLED"
        info["cuda_available"] = False
        info["warnings"].append("PyTorch is not installed.")

    info["triton_version"] = "not required"
    info["arch_list_set"] = bool(os.environ.get("TORCH_CUDA_ARCH_LIST", ""))
    info["sm120_ready"] = False
    info["sm100_ready"] = info.get("compute_cap") == "10.0"
    if info.get("cuda_available") and not info["sm100_ready"]:
        info["warnings"].append(
            f"GPU compute capability is {info.get('compute_cap')}; these kernels need sm_100 (B200)."
        )

    from ghostweight_triton_b200 import _native

    info["native_library"] = str(_native.LIB_PATH) if _native.LIB_PATH.exists() else "NOT BUILT"
    if not _native.LIB_PATH.exists():
        info["warnings"].append(
            "libghostweight_b200.so is not built: python -m ghostweight_triton_b200.csrc.build"
        )
    if verbose:
        _print_report(info)
    return info


def _print_report(info: dict) -> None:
    def mark(ok: bool) -> str:
        return "ok " if ok else "-- "

    print("\n  GhostWeight B200 environment check")
    print(f"  {mark(info.get('torch_version') != 'NOT INSTALLED')}PyTorch     {info.get('torch_version')}")
    print(f"  {mark(bool(info.get('cuda_available')))}CUDA        {info.get('cuda_version')}")
    print(f"  {mark(bool(info.get('cuda_available')))}GPU         {info.get('gpu_name')}")
    print(f"  {mark(bool(info.get('sm100_ready')))}Compute cap {info.get('compute_cap')}")
    print(f"  {mark(info.get('native_library') != 'NOT BUILT')}Native lib  {info.get('native_library')}")
    if info["warnings"]:
        print("\n  Warnings:")
        for w in info["warnings"]:
            print(f"    - {w}")
    else:
        print("\n  All checks passed.")
    print()
