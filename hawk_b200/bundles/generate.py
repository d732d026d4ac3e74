"""Regenerate the b200 bundles of the five benchmark kernels.

Traces the kernels of ``hawk_b200.configs`` with the reference's front end,
renders each b200 unit and compiles it with NVRTC for sm_100a, writing
``<kernel>.<mode>.cu`` / ``.cubin`` / ``.json`` here.  The units and sidecars
are committed; the CUBINs are rebuilt from the units by
``python -m hawk_b200.csrc.build``, which needs no front end.

``staged/`` holds the same units of two kernels built with their inputs
staged through shared memory (hk/stage.cuh) -- one lane-frame, one row-frame
entry -- so the staged path stays under the GPU parity tests although the
build policy picks it for no benchmark kernel today.

    python -m hawk_b200.bundles.generate
"""

from __future__ import annotations

from pathlib import Path

HERE = Path(__file__).resolve().parent
STAGED = HERE / "staged"
STAGED_KERNELS = ("spd_solve_vjp", "poly_loss_vjp")


def main() -> int:
    from hawk_b200 import configs
    from hawk_b200.target.build import build_kernel

    for name, (kernel, modes) in configs.KERNELS.items():
        for mode in modes:
            sidecar = build_kernel(kernel, HERE, name=name, mode=mode)
            regs = sidecar["b200"]["ptxas"].get(name, {})
            print(f"{name}.{mode}: frame={sidecar['b200']['frame']} regs={regs.get('regs')} "
                  f"stack={regs.get('stack_B')}")
    for name in STAGED_KERNELS:
        kernel, _modes = configs.KERNELS[name]
        sidecar = build_kernel(kernel, STAGED, name=name, mode="float64", staged=True)
        print(f"staged/{name}.float64: stages={sidecar['b200']['stages']} "
              f"smem={sidecar['b200']['dynamic_smem']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
