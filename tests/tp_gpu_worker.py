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


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    ok = True
    try:
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
            checks["no multicast"] = not graph_state.peers.multicast
            if rank == 0:
                print(case[0], checks, flush=True)
            ok = ok and all(checks.values())
    finally:
        dist.barrier()
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
