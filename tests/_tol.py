"""Tolerances of the parity suite (|got − ref| ≤ atol + rtol·|ref|, elementwise).

* fp32 inputs: rtol 1e-5, atol 1e-5 — the exact-fp32 CUDA-core path against a
  float64 oracle (fp32 round-off of HD-long dots and W-long sums stays well
  under 1e-5 for O(1) data).
* bf16 inputs: rtol 2e-2, atol 2e-2 — the tensor-core path (bf16 operands,
  fp32 accumulation, bf16 outputs) against the float64 oracle evaluated on the
  same bf16-rounded inputs.  For bf16 the absolute floor is taken relative to
  the tensor's scale: atol·max(1, rms(ref)).  Raw Σ τ·V outputs and some
  gradients have rms ≈ 3-6; there a fixed 2e-2 floor would demand better
  than the bf16 rounding of τ itself (2^-9 relative per term).  Unit-scale
  tensors (normalised outputs, τ) keep the plain 2e-2 floor.
"""
import numpy as np
import torch

TOL = {
    torch.float32: dict(rtol=1e-5, atol=1e-5),
    torch.bfloat16: dict(rtol=2e-2, atol=2e-2),
    torch.float16: dict(rtol=1e-2, atol=1e-2),
}


def assert_close(got, ref, dtype, what=""):
    g = got.detach().to(torch.float64).cpu()
    r = ref.detach().to(torch.float64).cpu() if isinstance(ref, torch.Tensor) else torch.from_numpy(np.asarray(ref, dtype=np.float64))
    tol = TOL[dtype]
    assert g.shape == r.shape, f"{what}: shape {tuple(g.shape)} vs {tuple(r.shape)}"
    err = (g - r).abs()
    atol = tol["atol"]
    if dtype in (torch.bfloat16, torch.float16):
        atol = atol * max(1.0, float(r.pow(2).mean().sqrt()))
    bound = atol + tol["rtol"] * r.abs()
    bad = err > bound
    if bad.any():
        idx = tuple(int(i) for i in torch.nonzero(bad)[0])
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.numel()} elements out of tolerance "
            f"{tol}; max err {float(err.max()):.3e}; first bad {idx}: "
            f"got {float(g[idx]):.6e} ref {float(r[idx]):.6e}")
