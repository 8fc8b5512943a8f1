"""Small, self-contained programs to run under a profiler: one case of one
kernel, a few launches, nothing else.

    python -m gb300_microbench_b200.profile_cases gemm M N K VARIANT [out_dtype]
    python -m gb300_microbench_b200.profile_cases copy METHOD STAGES BIF_KIB ROW_BYTES MIB
    python -m gb300_microbench_b200.profile_cases umma CTA_GROUP N DEPTH ITERATIONS
    python -m gb300_microbench_b200.profile_cases lowp KIND M N K [CTA_GROUP]

gemm: N(0,1) BF16 operands (torch.Generator seed 0), 4 launches of the plan.
copy: a MIB-MiB seeded uniform-u32 buffer, 3 one-pass launches.
umma: the reference's integer operands, 2 launches.
lowp: KIND nvfp4 or fp8_block128, quantised N(0,1) operands (seed 0),
      4 launches of the block-scaled plan (CTA_GROUP 1 or 2 forces the tile).
Each prints "ok" and exits 0 when the kernel reported no device error.
"""
from __future__ import annotations

import sys


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    import torch

    if not argv:
        print(__doc__)
        return 2
    what, args = argv[0], argv[1:]
    if what == "gemm":
        from .gemm import GemmPlan

        m, n, k = (int(x) for x in args[:3])
        variant = args[3] if len(args) > 3 else "tuned"
        out = torch.float32 if len(args) > 4 and args[4] == "f32" else torch.bfloat16
        g = torch.Generator().manual_seed(0)
        a = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
        b = torch.randn(n, k, generator=g).to(torch.bfloat16).cuda()
        c = torch.empty(m, n, dtype=out, device="cuda")
        plan = GemmPlan(a, b, c, variant=variant)
        plan.run(4)
        plan.synchronize()
    elif what == "copy":
        from . import streaming

        method, stages, bif, row_bytes, mib = args[0], int(args[1]), int(args[2]), int(args[3]), int(args[4])
        buf = torch.empty(mib * 1024 * 1024 // 4, dtype=torch.int32, device="cuda")
        streaming.fill_uniform_u32(buf)
        run = streaming.StreamingRun(method, stages, bif, buf, row_bytes=row_bytes)
        for _ in range(3):
            run.run()
        run.checksums()
        run.check_status()
    elif what == "umma":
        from . import inputs, umma

        cg, n, depth, iters = (int(x) for x in args[:4])
        a, b = inputs.umma_pattern_operands(cg, n)
        probe = umma.UmmaProbe(cg, n, depth, a.cuda(), b.cuda())
        for _ in range(2):
            probe.launch(iters)
        probe.result()
    elif what == "lowp":
        import os

        from . import lowp

        kind, (m, n, k) = args[0], (int(x) for x in args[1:4])
        if len(args) > 4:
            os.environ["BB_LOWP_CTA_GROUP"] = args[4]
        x, y = lowp.config4_inputs(m, n, k, seed=0, device="cuda")
        op = lowp.Nvfp4Operand if kind == "nvfp4" else lowp.Fp8BlockOperand
        a, b = op(x), op(y)
        del x, y
        d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        plan = lowp.LowpGemmPlan(kind, a, b, d)
        plan.run(4)
        plan.synchronize()
    else:
        print(__doc__)
        return 2
    print("ok")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
