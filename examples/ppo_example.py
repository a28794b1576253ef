"""PPO on vectorized CartPole with the turbol_b200 engines.

Same command line as the reference example (turbol_vllm/examples/py/ppo_example.py:31-46):
    python examples/ppo_example.py --num-envs 256 --rollout-steps 32 --batch-size 64 --num-updates 200

Where the reference steps a linear environment with random actions and updates
a linear policy on an uninitialised batch (ppo_example.py:150-185), this runs
the algorithm the flags describe: CartPole (obs_dim 4, 2 discrete actions,
auto-reset), an actor-critic MLP (tanh, orthogonal init), GAE(0.99, 0.95),
clipped PPO for 4 epochs of minibatches, Adam.  Every rollout step is also
pushed into a RingBuffer (capacity 8192 by default) as the reference does.

The default compute dtype is fp32 (the 256-env workload's precision): on a
GPU the environment, sampling, GAE, minibatch gather, loss and Adam run as
sm_100a kernels under CUDA graphs with an fp32 MLP; ``--dtype bf16`` switches
the MLP to the tensor-core path of the large-batch benchmark; on CPU the same
math in PyTorch.
Multi-GPU data parallel: ``torchrun --nproc-per-node N examples/ppo_example.py --dp fused``.
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile
import time

import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))

import turbol_b200 as turbol  # noqa: E402
from turbol_b200.rl.ppo import PPOConfig, PPOTrainer  # noqa: E402


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="turbol_b200 PPO example")
    p.add_argument("--num-envs", type=int, default=256, help="parallel environments (per GPU)")
    p.add_argument("--obs-dim", type=int, default=4, help="observation dimension (CartPole: 4)")
    p.add_argument("--act-dim", type=int, default=2, help="action count (CartPole: 2)")
    p.add_argument("--rollout-steps", type=int, default=32, help="steps per rollout")
    p.add_argument("--batch-size", type=int, default=64, help="minibatch size")
    p.add_argument("--num-updates", type=int, default=200, help="PPO iterations")
    p.add_argument("--lr", type=float, default=3e-4)
    p.add_argument("--device", type=str, default="cuda:0", help="cpu or cuda:N")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--log-dir", type=str, default="", help="TensorBoard/Prometheus directory (temp dir if empty)")
    p.add_argument("--print-every", type=int, default=20)
    # additions
    p.add_argument("--hidden", type=int, nargs="+", default=[64, 64])
    p.add_argument("--epochs", type=int, default=4)
    p.add_argument("--buffer-capacity", type=int, default=8192)
    p.add_argument("--dtype", choices=["bf16", "fp32"], default="fp32",
                   help="compute dtype: fp32 (the default, as in the 256-env CartPole workload) or bf16 (the "
                        "tensor-core path of the large-batch benchmark)")
    p.add_argument("--dp", choices=["none", "nccl", "fused"], default="none",
                   help="data parallel gradient reduction (launch with torchrun)")
    p.add_argument("--checkpoint-dir", type=str, default="")
    p.add_argument("--checkpoint-every", type=int, default=0)
    p.add_argument("--resume", action="store_true", help="resume from the latest checkpoint in --checkpoint-dir")
    return p.parse_args(argv)


def main(argv=None):
    args = parse_args(argv)
    if (args.obs_dim, args.act_dim) != (4, 2):
        raise SystemExit("this example trains CartPole: --obs-dim 4 --act-dim 2")
    if args.device.startswith("cuda") and not torch.cuda.is_available():
        args.device = "cpu"
    world, rank = int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("RANK", 0))
    group = None
    if args.dp != "none" and world > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", 0))
        args.device = f"cuda:{local}"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    else:
        args.dp = "none"
    cfg = PPOConfig(num_envs=args.num_envs, rollout_steps=args.rollout_steps, hidden=tuple(args.hidden),
                    epochs=args.epochs, minibatch_size=args.batch_size, lr=args.lr, seed=args.seed,
                    compute_dtype=args.dtype if args.device.startswith("cuda") else "fp32")
    tr = PPOTrainer(cfg, device=args.device, rank=rank, dp=args.dp, group=group)
    start = 0
    from turbol_b200.utils.checkpoint import latest_step

    if args.resume and args.checkpoint_dir and latest_step(args.checkpoint_dir) is not None:
        st = turbol.load_checkpoint(args.checkpoint_dir, trainer=tr)
        start = st["step"]
        print(f"resumed from step {start}")

    log_dir = args.log_dir or tempfile.mkdtemp(prefix="turbol_ppo_")
    os.makedirs(log_dir, exist_ok=True)
    tb = turbol.TensorBoardWriter(log_dir) if rank == 0 else None
    prom = turbol.PrometheusWriter(os.path.join(log_dir, "metrics.prom")) if rank == 0 else None
    prof = turbol.Profiler()
    prof.enable()
    buf = turbol.RingBuffer(args.buffer_capacity, args.obs_dim, 1, "cuda" if tr.cuda else "cpu")
    if rank == 0:
        print(f"PPO CartPole: {cfg.num_envs} envs x {cfg.rollout_steps} steps, MLP 4-{'-'.join(map(str, cfg.hidden))}, "
              f"{cfg.epochs} epochs x minibatch {cfg.minibatch_size}, device {args.device}, dp {args.dp} x {world}")
    steps_per_iter = tr.env_steps_per_iteration() * (world if args.dp != "none" else 1)
    for it in range(start, args.num_updates):
        t0 = time.perf_counter()
        with prof.span("iteration", "train"):
            tr.train_iteration()
            # the iteration's transitions go into the replay ring, as in the reference loop
            T = cfg.rollout_steps
            obs = tr.obs_buf.view(T * cfg.num_envs, 4)
            act = tr.act_buf.view(-1, 1).float()
            ft = turbol.from_torch
            st = buf.push_batch(ft(obs), ft(act), ft(tr.rew_buf.view(-1)), ft(tr.done_buf.view(-1).bool()))
            if not st.ok():
                raise RuntimeError(f"push_batch: {st}")
        if tr.cuda:
            torch.cuda.synchronize(tr.device)
        dt = time.perf_counter() - t0
        if (it + 1) % args.print_every == 0 or it + 1 == args.num_updates:
            m = tr.metrics()
            fps = steps_per_iter / dt
            if rank == 0:
                print(f"update {it + 1:5d}  return {m['mean_return']:8.2f}  len {m['mean_length']:7.1f}  "
                      f"pi_loss {m['policy_loss']:+.4f}  v_loss {m['value_loss']:.4f}  kl {m['approx_kl']:.4f}  "
                      f"fps {fps:,.0f}  buffer {buf.size()}")
                for k, v in (("train/mean_reward", m["mean_return"]), ("train/fps", fps),
                             ("train/policy_loss", m["policy_loss"]), ("train/value_loss", m["value_loss"]),
                             ("train/entropy", m["entropy"]), ("train/approx_kl", m["approx_kl"]),
                             ("train/clipfrac", m["clipfrac"]), ("buffer/size", float(buf.size())),
                             ("time/iteration_ms", dt * 1e3)):
                    if v == v:  # skip NaN (no finished episode yet)
                        tb.add_scalar(k, float(v), it + 1)
                prom.write_gauge("turbol_ppo_fps", float(fps))
                prom.write_gauge("turbol_ppo_mean_return",
                                 float(m["mean_return"]) if m["mean_return"] == m["mean_return"] else 0.0)
                prom.flush()
        if args.checkpoint_dir and args.checkpoint_every and (it + 1) % args.checkpoint_every == 0:
            # every rank writes its own files (environments, RNG, optimizer shard)
            turbol.save_checkpoint(args.checkpoint_dir, it + 1, tr, background=False, keep_last=3)
    if rank == 0:
        tb.flush()
        prof.export_chrome_trace(os.path.join(log_dir, "trace.json"))
        print(f"logs: {log_dir}")
    if args.dp != "none":
        import torch.distributed as dist

        tr.release_graphs()
        dist.destroy_process_group()
    return tr


if __name__ == "__main__":
    main()
