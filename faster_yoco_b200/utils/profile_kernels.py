"""Small, self-terminating launches of the hot kernels for `ncu` captures (a few MB on the device, a handful of
launches each). Used as:  ncu --set full --clock-control none -k regex:<kernel> -s <n> -c <m> \\
    python -m faster_yoco_b200.utils.profile_kernels --what attn|ret|gemm|attn_bwd|ret_bwd|norm|ce|adam
"""
import argparse

import torch


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--what", default="attn")
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--L", type=int, default=2048)
    a = p.parse_args()
    from faster_yoco_b200 import ops
    C = ops._C()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    L = a.L
    if a.what in ("attn", "attn_bwd"):
        q = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        k = torch.randn(1, L, 8, 128, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, L, 8, 128, device=dev, dtype=torch.bfloat16)
        o, lse = C.attention_fwd(q, k, v, True, 0, 128 ** -0.5)
        do = torch.randn_like(o)
        for _ in range(a.reps):
            if a.what == "attn":
                C.attention_fwd(q, k, v, True, 0, 128 ** -0.5)
            else:
                C.attention_bwd(do, q, k, v, o, lse, True, 0, 128 ** -0.5)
    elif a.what in ("ret", "ret_bwd"):
        q = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        k = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        g = (torch.nn.functional.logsigmoid(torch.randn(1, 24, L, device=dev)) / 16).cumsum(-1).contiguous()
        o = C.retention_fwd(q, k, v, g)
        do = torch.randn_like(o)
        for _ in range(a.reps):
            if a.what == "ret":
                C.retention_fwd(q, k, v, g)
            else:
                C.retention_bwd(do, q, k, v, g, o)
    elif a.what == "gemm":
        x = torch.randn(2048, 3072, device=dev, dtype=torch.bfloat16)
        w = torch.randn(12312, 3072, device=dev, dtype=torch.bfloat16)
        y = torch.empty(2048, 12312, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            C.gemm(x, w, y, False, False, None)
    elif a.what == "gemm_dgrad":
        dy = torch.randn(2048, 16384, device=dev, dtype=torch.bfloat16)
        w = torch.randn(16384, 3072, device=dev, dtype=torch.bfloat16)
        y = torch.empty(2048, 3072, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            C.gemm(dy, w, y, False, True, None)
    elif a.what == "adam":
        # a quarter of one rank's ZeRO segment at 8 GPUs (1.7 GB in total, well above L2)
        n = 107_665_728
        p32 = torch.randn(n, device=dev)
        m = torch.zeros(n, device=dev)
        v = torch.zeros(n, device=dev)
        g16 = torch.randn(n, device=dev, dtype=torch.bfloat16)
        p16 = torch.empty(n, device=dev, dtype=torch.bfloat16)
        hyper = torch.tensor([1e-4, 0.1, 0.05, 0.0], device=dev)
        factor = torch.tensor([1.0], device=dev)
        for _ in range(a.reps):
            C.adam_step(p32, g16, m, v, p16, hyper, factor, 0.9, 0.95, 1e-6, 0.05, True)
    elif a.what in ("ce", "ce_bwd"):
        x = (torch.randn(L, 100288, device=dev) * 2).to(torch.bfloat16)
        t = torch.randint(0, 100288, (L,), device=dev)
        loss, lse = C.ce_fwd(x, t, 1)
        g = torch.ones(1, device=dev)
        out = torch.empty_like(x)
        for _ in range(a.reps):
            if a.what == "ce":
                C.ce_fwd(x, t, 1)
            else:
                C.ce_bwd(x, t, lse, g, 1, out)
    elif a.what in ("rms", "rms_bwd"):
        x = torch.randn(L, 3072, device=dev, dtype=torch.bfloat16)
        w = torch.ones(3072, device=dev, dtype=torch.bfloat16)
        y, rstd = C.rms_norm_fwd(x, w, 1e-5)
        for _ in range(a.reps):
            if a.what == "rms":
                C.rms_norm_fwd(x, w, 1e-5)
            else:
                C.rms_norm_bwd(y, x, w, rstd)
    else:
        raise SystemExit(f"unknown --what {a.what}")
    torch.cuda.synchronize()
    st = int(C.status()[0].item())
    if st != 0:
        raise SystemExit(f"device status {st:#x}")


if __name__ == "__main__":
    main()
