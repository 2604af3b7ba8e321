"""Tensor-parallel building blocks on N ranks with the multi-process executor: a
column-parallel -> row-parallel MLP whose sharded output equals the unsharded one.

    python examples/tp_layers_mpexecutor.py --world-size 2            # CPU, gloo
    python examples/tp_layers_mpexecutor.py --world-size 2 --cuda     # one GPU per rank, NCCL

Each rank loads its slice of the full weights through the parameters' ``weight_loader``
(columns of the first layer, rows of the second) and the row-parallel layer sums the partial
products with an all-reduce.
"""

import argparse

import torch


def _full_weights(h: int, f: int):
    g = torch.Generator().manual_seed(0)
    return torch.randn(f, h, generator=g) / h ** 0.5, torch.randn(h, f, generator=g) / f ** 0.5


def build(ctx, h, f):
    from vllm_neuron_b200.nn.linear import ColumnParallelLinear, RowParallelLinear

    w1, w2 = _full_weights(h, f)
    up = ColumnParallelLinear(h, f, ctx.ps.tp, bias=False, dtype=torch.float32, device=ctx.device)
    down = RowParallelLinear(f, h, ctx.ps.tp, bias=False, dtype=torch.float32, device=ctx.device)
    up.weight.weight_loader(up.weight, w1.to(ctx.device))
    down.weight.weight_loader(down.weight, w2.to(ctx.device))
    return up, down


def forward(ctx, x):
    up, down = ctx.obj
    with torch.no_grad():
        return down(torch.relu(up(x.to(ctx.device)))).cpu()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--world-size", type=int, default=2)
    ap.add_argument("--cuda", action="store_true")
    ap.add_argument("--hidden", type=int, default=256)
    ap.add_argument("--ffn", type=int, default=1024)
    a = ap.parse_args()
    from vllm_neuron_b200.utils.executor import MPExecutor

    x = torch.randn(8, a.hidden)
    w1, w2 = _full_weights(a.hidden, a.ffn)
    want = torch.relu(x @ w1.T) @ w2.T
    with MPExecutor(world_size=a.world_size, tp=a.world_size, backend="nccl" if a.cuda else "gloo") as ex:
        ex.load(build, a.hidden, a.ffn)
        outs = ex.run(forward, x)
    for r, y in enumerate(outs):
        print(f"rank {r}: max |diff| vs unsharded = {(y - want).abs().max():.2e}")
    assert all(torch.allclose(y, want, atol=1e-4) for y in outs)
    print("ok")


if __name__ == "__main__":
    main()
