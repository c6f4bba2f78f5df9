"""Named single-kernel cases of the hot path, sized for profiling.

``python -m einsum_ir_b200.profile_cases <case|all> [--reps N] [--time]``
runs each case through the C-ABI: one untimed launch, then N launches
(default 1). With ``--time`` it prints one JSON line per case with the CUDA
event time per launch and the achieved rate against the algorithmic work
(permutes: 2 x tensor bytes moved; contractions: 2|C||M||N||K| flop). The
cases keep well under a few GB on the device (every operand still larger
than the 126 MB L2), so an ncu capture of them ends in a minute or two:

  permute_transpose  FP32 [8192][8192] -> [8192][8192]^T (256 MiB each way)
  permute_copy4d     FP32 96^4, abcd -> acbd (rows of d copied, 324 MiB)
  tf32_slab          BASELINE config 5 with z = 8, TF32 (two TF32-rounding
                     operand copies + the CTA-pair tcgen05 kernel)
  fp32x3_slab        the same in FP32-exact mode (3xTF32 CTA-pair kernel)
  fp64_slab          the same in FP64 (DMMA kernel)
  bf16_cfg2          BASELINE config 2 (pre-permute + BF16 CTA-pair kernel)
  bf16_mlp_layer     BASELINE config 3, one layer: bi,io->bo, b = 8192, widths 4096, BF16,
                     COPY bias (broadcast over b) first touch, RELU last touch
  readme_tree        BASELINE config 1: the README expression iae,bf,dcba,cg,dh->hgfei through
                     eir_expression (FP32; the second and later evaluations replay a CUDA graph)
  tucker             BASELINE config 4: abc,ia,jb,kc->ijk, core 128^3, factors 1024 x 128, path
                     (0,1),(0,2),(0,1), FP32 through eir_expression (4.29 GB output: a few GB on
                     the device, too large for an ncu capture; time it with --time)
"""
from __future__ import annotations

import json
import sys

from . import binary, cabi


def _contraction(expr, sizes, dt, comp=cabi.COMPUTE_DEFAULT, bias_bcast=None):
    import torch
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    dto = cabi.FP64 if dt == cabi.FP64 else cabi.FP32
    aux_sizes = None if bias_bcast is None else {i: (1 if names[i] == bias_bcast else sz[i]) for i in sz}
    touch = (cabi.KTYPE_ZERO, cabi.KTYPE_UNDEFINED) if aux_sizes is None else (cabi.KTYPE_COPY, cabi.KTYPE_RELU)
    plan = cabi.ContractPlan(binary.contraction_dims(il, ir, io, sz, sizes_outer_aux=aux_sizes), dt, dt, dto,
                             comp, touch[0], cabi.KTYPE_MADD, touch[1])
    tdt = {cabi.FP64: torch.float64, cabi.BF16: torch.bfloat16}.get(dt, torch.float32)
    g = torch.Generator(device="cuda").manual_seed(0)
    l = (torch.rand([sz[i] for i in il], generator=g, device="cuda") * 2 - 1).to(tdt)
    r = (torch.rand([sz[i] for i in ir], generator=g, device="cuda") * 2 - 1).to(tdt)
    o = torch.empty([sz[i] for i in io], device="cuda",
                    dtype=torch.float64 if dto == cabi.FP64 else torch.float32)
    aux = None if aux_sizes is None else torch.rand([aux_sizes[i] for i in io], generator=g, device="cuda",
                                                   dtype=o.dtype)
    return (lambda: plan.contract(l, r, o, aux)), plan.num_ops, "flop", plan.describe()


def _readme_tree():
    return _expression("iae,bf,dcba,cg,dh->hgfei", "32,8,4,2,16,64,8,8,8", "(1,2),(2,3),(0,1),(0,1)")


def _tucker():
    return _expression("abc,ia,jb,kc->ijk", "128,128,128,1024,1024,1024", "(0,1),(0,2),(0,1)")


def _expression(expr, sizes, path):
    import torch
    e = cabi.Expression(expr, sizes, path, cabi.FP32)
    g = torch.Generator(device="cuda").manual_seed(0)
    ts = [torch.rand(e.tensor_shape(i), generator=g, device="cuda") * 2 - 1 for i in range(e.num_tensors)]
    st = torch.cuda.Stream()  # graph replay needs a non-default stream
    torch.cuda.current_stream().wait_stream(st)

    def fn():
        with torch.cuda.stream(st):
            e.eval(ts, stream=st.cuda_stream)
        torch.cuda.current_stream().wait_stream(st)
    return fn, e.num_ops, "flop", e.describe()


def _permute(shape, perm):
    import torch
    x = torch.rand(shape, device="cuda")
    y = torch.empty([shape[i] for i in perm], device="cuda")
    # strides of every input dim in the input and in the output
    sin = list(x.stride())
    pos = {d: k for k, d in enumerate(perm)}
    sout = [y.stride()[pos[d]] for d in range(len(shape))]
    plan = cabi.PermutePlan(list(shape), sin, sout, cabi.FP32)
    return (lambda: plan.permute(x, y)), 2 * x.numel() * 4, "bytes", plan.describe()


CASES = {
    "permute_transpose": lambda: _permute((8192, 8192), (1, 0)),
    "permute_copy4d": lambda: _permute((96, 96, 96, 96), (0, 2, 1, 3)),
    "tf32_slab": lambda: _contraction("zabcd,zcdef->zabef", dict(z=8, a=48, b=48, c=48, d=48, e=48, f=48),
                                      cabi.FP32, cabi.COMPUTE_TF32),
    "fp32x3_slab": lambda: _contraction("zabcd,zcdef->zabef", dict(z=8, a=48, b=48, c=48, d=48, e=48, f=48),
                                        cabi.FP32),
    "fp64_slab": lambda: _contraction("zabcd,zcdef->zabef", dict(z=8, a=48, b=48, c=48, d=48, e=48, f=48),
                                      cabi.FP64),
    "bf16_cfg2": lambda: _contraction("akmj,njk->anm", dict(a=16, k=32, m=512, j=64, n=512), cabi.BF16),
    "bf16_mlp_layer": lambda: _contraction("bi,io->bo", dict(b=8192, i=4096, o=4096), cabi.BF16,
                                           bias_bcast="b"),
    "readme_tree": _readme_tree,
    "tucker": _tucker,
}


def run(name: str, reps: int, timed: bool) -> dict | None:
    import torch
    fn, work, unit, desc = CASES[name]()
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    cabi.check_device_errors()
    ms = e0.elapsed_time(e1) / max(1, reps)
    rate = work / (ms * 1e-3) / (1e9 if unit == "bytes" else 1e12)
    res = {"case": name, "ms_per_launch": ms, "rate": rate, "rate_unit": "GB/s" if unit == "bytes" else "TFLOP/s",
           "work": work, "work_unit": unit, "plan": desc}
    torch.cuda.empty_cache()
    return res if timed else None


def main(argv) -> int:
    names = [a for a in argv if not a.startswith("--")]
    reps = 1
    for a in argv:
        if a.startswith("--reps="):
            reps = int(a.split("=", 1)[1])
    if not names or names == ["all"]:
        names = list(CASES)
    for n in names:
        res = run(n, reps, "--time" in argv)
        if res is not None:
            print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
