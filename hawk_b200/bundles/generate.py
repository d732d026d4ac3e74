"""Regenerate the b200 bundles of the five benchmark kernels.

Traces the kernels of ``hawk_b200.configs`` with the reference's front end,
renders each b200 unit and compiles it with NVRTC for sm_100a, writing
``<kernel>.<mode>.cu`` / ``.cubin`` / ``.json`` here.  The units and sidecars
are committed; the CUBINs are rebuilt from the units by
``python -m hawk_b200.csrc.build``, which needs no front end.

    python -m hawk_b200.bundles.generate
"""

from __future__ import annotations

from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> int:
    from hawk_b200 import configs
    from hawk_b200.target.build import build_kernel

    for name, (kernel, modes) in configs.KERNELS.items():
        for mode in modes:
            sidecar = build_kernel(kernel, HERE, name=name, mode=mode)
            regs = sidecar["b200"]["ptxas"].get(name, {})
            print(f"{name}.{mode}: frame={sidecar['b200']['frame']} regs={regs.get('regs')} "
                  f"stack={regs.get('stack_B')}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
