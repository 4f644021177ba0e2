"""torchrun worker for tests/test_tp_gpu.py: the tiny Qwen3 through the B200 engine at TP = world
size (NCCL all-reduce after o_proj and down_proj, eager and inside the captured graph)."""

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


def check_push_forms(comm, device, rank, world):
    """Every all-reduce form through the add+RMSNorm consumer: split partials + the fused push /
    all-reduce / add+RMSNorm kernel (the decode default), split partials + fb_reduce_push +
    fb_allreduce_add_rmsnorm, the projection's push epilogue at one split and with its K splits
    summed by the split fix-up. Every rank gets the same bits, forms over the same K splits
    agree bit for bit, and all are close to an NCCL all-reduce of the fp32 partials followed
    by the same add + RMSNorm."""
    from kernels import linear as klinear
    from kernels._native import check, lib, ptr, stream
    from kernels.rmsnorm import add_rms_norm
    forms = (("fused", 512, None), ("one split", 512, 1), ("fix-up", 512, None),
             ("fused", 1536, None), ("reduce-push", 1536, None), ("fix-up", 1536, None))
    peers = fdecode.PeerBuffers(comm, len(forms), 16, 4096, device)
    epoch = torch.full((1,), 41, dtype=torch.int64, device=device)
    g = torch.Generator(device=device).manual_seed(100 + rank)
    residual = torch.randn(16, 4096, device=device, generator=torch.Generator(device=device).manual_seed(7)).bfloat16()
    gain = torch.ones(4096, device=device).bfloat16()
    checks, outs, inputs = {}, {}, {}
    for use, (form, k, splits) in enumerate(forms):
        if k not in inputs:
            inputs[k] = (torch.randn(16, k, device=device, generator=g).bfloat16(),
                         (torch.randn(4096, k, device=device, generator=g) * 0.05).bfloat16())
        x, weight = inputs[k]
        if form == "reduce-push":
            s = klinear.splits_for(16, 4096, k, device)
            part = klinear.project(x, weight, klinear.SPLITS_OUT, s)
            check(lib.fb_reduce_push(ptr(part), s, 16, 4096, world, rank, use, peers.recv_ptrs, peers.mc_ptr,
                                     ptr(epoch), stream()), "fb_reduce_push")
            out, summed = torch.empty_like(residual), torch.empty_like(residual)
            check(lib.fb_allreduce_add_rmsnorm(peers.recv_local, use, world, ptr(epoch), ptr(residual), ptr(gain),
                                               ptr(out), ptr(summed), 16, 4096, 1e-6, stream()),
                  "fb_allreduce_add_rmsnorm")
        else:
            out, summed = fdecode._allreduce_add_norm(x, weight, comm, peers, use, epoch, residual, gain, 1e-6,
                                                      split_consumer=form == "fused", splits=splits)
        partial = x.float() @ weight.float().T
        dist.all_reduce(partial)
        ref_out, ref_sum = add_rms_norm(partial.bfloat16(), residual, gain, 1e-6)
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        name = f"K={k} {form}"
        outs[name] = (out, summed)
        checks[f"{name} ranks agree"] = all(torch.equal(t, gathered[0]) for t in gathered)
        checks[f"{name} vs NCCL"] = bool((out.float() - ref_out.float()).abs().max() <= 0.05) and \
            bool((summed.float() - ref_sum.float()).abs().max() <= 0.05)
    for k in (512, 1536):
        same = [outs[f"K={k} fused"], outs[f"K={k} fix-up"]] + ([outs["K=1536 reduce-push"]] if k == 1536 else [])
        checks[f"K={k} split forms equal"] = all(torch.equal(a[0], same[0][0]) and torch.equal(a[1], same[0][1])
                                                 for a in same)
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
        push_checks = check_push_forms(comm0, device, rank, world)
        if rank == 0:
            print("push forms", push_checks, "multicast" if os.environ.get("FB_TP_MULTICAST", "0") == "1" else "peer stores",
                  flush=True)
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
            if os.environ.get("FB_TP_MULTICAST", "0") != "1":
                checks["no multicast"] = not graph_state.peers.multicast
            else:
                checks["multicast used"] = graph_state.peers.multicast
            if rank == 0:
                print(case[0], checks, flush=True)
            ok = ok and all(checks.values())
    finally:
        dist.barrier()
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
