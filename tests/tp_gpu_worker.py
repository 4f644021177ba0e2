"""torchrun worker for tests/test_tp_gpu.py: the tiny Qwen3 through the B200 engine at TP = world
size (the flagged-word NVLink all-reduce after o_proj and down_proj, eager and inside the captured
graph; NCCL all-reduces in the eager prefill)."""

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, os.path.join(ROOT, "fast-transformer_b200"), os.path.join(HERE, "golden")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import cases  # noqa: E402
import decode as fdecode  # noqa: E402
import qwen3  # noqa: E402


def check_allreduce(comm, device, rank, world, form):
    """The decode step's all-reduce in one of its forms (push: fb_allreduce_push +
    fb_allreduce_sum_add_rmsnorm; owner: fb_reduce_scatter_push + fb_allreduce_add_rmsnorm) over
    the projection's split partials, at two K widths (different split counts): every rank gets
    the same bits, close to an NCCL all-reduce of the fp32 partials followed by the same
    add + RMSNorm."""
    from kernels.rmsnorm import add_rms_norm
    widths = (512, 1536)
    peers = fdecode.PeerBuffers(comm, len(widths), 16, 4096, device, form=form)
    epoch = torch.full((1,), 41, dtype=torch.int64, device=device)
    g = torch.Generator(device=device).manual_seed(100 + rank)
    residual = torch.randn(16, 4096, device=device, generator=torch.Generator(device=device).manual_seed(7)).bfloat16()
    gain = torch.ones(4096, device=device).bfloat16()
    checks = {}
    for use, k in enumerate(widths):
        x = torch.randn(16, k, device=device, generator=g).bfloat16()
        weight = (torch.randn(4096, k, device=device, generator=g) * 0.05).bfloat16()
        out, summed = fdecode._allreduce_add_norm(x, weight, comm, peers, use, epoch, residual, gain, 1e-6)
        partial = x.float() @ weight.float().T
        dist.all_reduce(partial)
        ref_out, ref_sum = add_rms_norm(partial.bfloat16(), residual, gain, 1e-6)
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        name = f"{form} K={k}"
        checks[f"{name} ranks agree"] = all(torch.equal(t, gathered[0]) for t in gathered)
        checks[f"{name} vs NCCL"] = bool((out.float() - ref_out.float()).abs().max() <= 0.05) and \
            bool((summed.float() - ref_sum.float()).abs().max() <= 0.05)
    torch.cuda.synchronize()
    return checks


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    ok = True
    try:
        comm0 = fdecode.Communicator(dist.group.WORLD, world, rank)
        push_checks = check_allreduce(comm0, device, rank, world, "push")
        push_checks.update(check_allreduce(comm0, device, rank, world, "owner"))
        if rank == 0:
            print("all-reduce", push_checks, flush=True)
        ok = all(push_checks.values())
        fx = torch.load(os.path.join(HERE, "golden", "model.pt"), weights_only=False)
        cfg = qwen3.Config.make(**cases.TINY_QWEN3)
        state_dict = cases.tiny_qwen3_weights()
        for case in cases.MODEL_CASES:
            prompt, steps = cases.model_prompt(case)
            batch, length = prompt.shape
            weights = qwen3.from_state_dict(cfg, state_dict, device, rank, world)
            comm = fdecode.Communicator(dist.group.WORLD, world, rank)
            eager = fdecode.DecodeState(weights, batch, length, steps + 4, comm=comm, device=device)
            tokens, logits = fdecode.greedy(eager, prompt.to(device), steps)
            graph_state = fdecode.DecodeState(weights, batch, length, steps + 4, comm=comm, device=device)
            graph_state.prefill(prompt.to(device))
            graphed = [graph_state.token_ids[:, 0].clone()]
            graph_state.capture()
            for _ in range(steps - 1):
                graph_state.step()
                graphed.append(graph_state.token_ids[:, 0].clone())
            torch.cuda.synchronize()
            graphed = torch.stack(graphed, 1)
            graph_state.release()
            gathered = [torch.empty_like(tokens) for _ in range(world)]
            dist.all_gather(gathered, tokens)
            expect = fx[case[0]]["native_tokens"].to(device)
            scale = fx[case[0]]["native_logits"].abs().max()
            err = (logits.cpu() - fx[case[0]]["native_logits"]).abs().max()
            checks = {
                "tokens == reference": torch.equal(tokens, expect),
                "graph == eager": torch.equal(graphed, tokens),
                "ranks agree": all(torch.equal(t, gathered[0]) for t in gathered),
                "logits": bool(err <= 2e-2 * scale),
            }
            if rank == 0:
                print(case[0], checks, flush=True)
            ok = ok and all(checks.values())
    finally:
        dist.barrier()
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
