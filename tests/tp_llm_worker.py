"""Worker for the tensor-parallel model test (2 GPUs, torchrun): the TP
forward (fused all-gather->GEMM / GEMM->reduce-scatter) matches the
single-GPU forward on each rank's rows, and TP greedy generation agrees with
single-GPU greedy generation."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.models.llm import DecoderLM, LMConfig  # noqa: E402
from turbol_b200.models.tp_llm import TPDecoderLM  # noqa: E402
from turbol_b200.parallel.tp import TensorParallelComm  # noqa: E402
from turbol_b200.rl.rollout import LLMGenerator, TPLLMGenerator  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = LMConfig.tiny(n_layers=2)
    cfg.init_std = 0.05
    full = DecoderLM(cfg, dev, seed=3, master=False)
    comm = TensorParallelComm(max_rows=4096, max_in=cfg.hidden, max_out=cfg.hidden)
    tpm = TPDecoderLM(full, comm)
    # ---- prefill forward
    P, Lp = 16, 64
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, cfg.vocab, (P, Lp), generator=g).to(dev, torch.int32)
    pos = torch.arange(Lp, device=dev, dtype=torch.int32).repeat(P)
    ref, _ = full.forward(full.embed(ids), P, Lp, pos)
    x = tpm.embed_rows(ids.reshape(-1))
    y = tpm.forward(x, P, Lp, pos)
    torch.cuda.synchronize()
    m = P * Lp // world
    exp = ref[rank * m:(rank + 1) * m].float()
    err = (y.float() - exp).abs().max().item() / (exp.abs().max().item() + 1e-6)
    assert err < 3e-2, ("forward", err)
    comm.check()
    # ---- greedy generation: TP vs single GPU
    P, Lp, G, new = 32, 32, 8, 12
    prompts = torch.randint(0, cfg.vocab, (P, Lp), generator=g).to(dev, torch.int32)
    gen1 = LLMGenerator(full, max_batch=P * G, max_len=Lp + new)
    s1, _ = gen1.generate(prompts, G, new, temperature=0.0)
    gen2 = TPLLMGenerator(tpm, max_batch=P * G, max_len=Lp + new)
    for rep in range(2):  # second call replays the captured step
        s2, lp2 = gen2.generate(prompts, G, new, temperature=0.0)
        torch.cuda.synchronize()
        agree = (s1[:, Lp:] == s2[:, Lp:]).float().mean().item()
        assert agree > 0.9, ("generate", rep, agree)
    s3, lp3 = gen2.generate(prompts, G, new, temperature=1.0)
    assert int(s3.max()) < cfg.vocab and bool(torch.all(lp3 <= 0))
    comm.check()
    if rank == 0:
        print("TP_LLM_WORKER_OK", err, agree)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
