"""The trainer's optimizer loop and the ``Train(model, dataset, config)`` surface
(crates/mmn-py/src/train/mod.rs:14-44 calling train_with_encoder,
crates/mmn-train/src/lib.rs:354-448) over the batched GPU step.

The reference's loop, restated: a HybridOptimizer (MuonConfig::default(),
AdamW with lr = learning_rate) and a separate AdamW are built once per run;
``optimizer == "hybrid"`` steps through the first, anything else (including
"muon") through the second. ``param_id`` grows by one per tensor per step and
is never reused, so m, v and velocity start at zero every step while the AdamW
step counter keeps counting. With ``batch_size == 1`` each sample is stepped
at once; otherwise each tensor's grads are summed over the micro-batches of a
batch (GradAccumulator) and averaged on the flush after ``batch_size``
micro-batches or at the last sample of an epoch (lib.rs:431).

Here the model's forward and backward stay with the caller: ``model`` supplies
its tensors in optimizer call order and one sample's grads, and each flush is
one ``mmn_optim_step_host`` call that divides by the micro-batch count on the
GPU and writes the updated fp32 weights back into the model's arrays.
"""
from __future__ import annotations

from typing import Callable, Protocol, Sequence

import numpy as np

from .step import OptimizerStep, TrainConfig, step_config_for


class TrainModel(Protocol):
    """What the loop needs from a model: its trained tensors in the order the
    optimizer visits them (e.g. ``chatbot_param_order``), their host arrays
    (updated in place), and the grads of one sample (same shapes, fp32)."""

    def param_order(self) -> Sequence[tuple[str, tuple[int, ...]]]: ...

    def parameters(self) -> Sequence[np.ndarray]: ...

    def backward(self, sample) -> Sequence[np.ndarray]: ...


class TrainLoop:
    """train_with_encoder's optimizer plumbing (lib.rs:382-442) over any stepper
    with ``step_host(grads, params, grad_divisor)`` and ``len(shapes)``
    tensors: the GPU ``OptimizerStep`` in the product, a per-call oracle replay
    in the tests."""

    def __init__(self, config: TrainConfig, step, shapes):
        self.config = config
        self.step = step
        self.shapes = [tuple(s) for s in shapes]
        self.param_id = 0
        self.steps = 0

    def run(self, n_samples: int, order: Callable[[int], Sequence[int]],
            backward: Callable[[int], Sequence[np.ndarray]], params: list[np.ndarray]) -> None:
        n = len(self.shapes)
        if len(params) != n:
            raise ValueError(f"need {n} parameter arrays (one per tensor)")
        batch_size = max(self.config.batch_size, 1)  # lib.rs:381
        for epoch in range(self.config.epochs):
            idx = list(order(epoch))
            if len(idx) != n_samples:
                raise ValueError("the epoch order must list every sample once")
            sums = None  # GradAccumulator, a new one per epoch (lib.rs:390)
            micro = 0
            for i, sample in enumerate(idx):
                grads = [np.ascontiguousarray(g, np.float32) for g in backward(sample)]
                if len(grads) != n or any(g.shape != s for g, s in zip(grads, self.shapes)):
                    raise ValueError("backward must return one grad per tensor, same shapes")
                if batch_size == 1:  # train_step_lm without an accumulator
                    self.step.step_host(grads, params, 1.0)
                    self.param_id += n
                    self.steps += 1
                    continue
                micro += 1
                if sums is None:
                    sums = [g.copy() for g in grads]
                else:
                    for acc, g in zip(sums, grads):
                        acc += g  # fp32, micro-batch order (lib.rs:246-248)
                if micro >= batch_size or i + 1 == len(idx):  # lib.rs:431
                    self.step.step_host(sums, params, float(micro))
                    self.param_id += n
                    self.steps += 1
                    sums = None
                    micro = 0


def train_loop(config: TrainConfig, param_order, params: list[np.ndarray],
               backward: Callable[[int], Sequence[np.ndarray]], n_samples: int,
               order: Callable[[int], Sequence[int]] | None = None, seed: int | None = None,
               device: int = 0) -> TrainLoop:
    """Runs the trainer's optimizer loop on the GPU. ``param_order`` is the
    (name, shape) list in call order; ``params`` the matching fp32 host arrays,
    updated in place; ``backward(sample)`` returns one sample's grads.
    ``order(epoch)`` gives an epoch's sample order; without it the samples are
    shuffled as lib.rs:385-389 does, from ``seed`` (None: fresh entropy, like
    the reference's thread_rng)."""
    cfg = step_config_for(config)  # the CUDA gate: cuda without a GPU raises CUDAError
    if not config.cuda:
        raise ValueError("cuda=False trains with the reference's CPU optimizer; this library "
                         "steps on the GPU (TrainConfig(cuda=True))")
    shapes = [tuple(s) for _, s in param_order]
    step = OptimizerStep([(k, s) for k, s in enumerate(shapes)], cfg, device=device)
    try:
        for k, p in enumerate(params):
            step.set_param(k, p)
        if order is None:
            rng = np.random.default_rng(seed)

            def order(_epoch):
                idx = list(range(n_samples))
                for i in range(n_samples):  # swap with a uniformly drawn index
                    j = int(rng.integers(0, n_samples))
                    idx[i], idx[j] = idx[j], idx[i]
                return idx

        loop = TrainLoop(config, step, shapes)
        loop.run(n_samples, order, backward, params)
        loop.adamw_step = step.adamw_step
        return loop
    finally:
        step.close()


def Train(model: TrainModel, dataset, config: TrainConfig, seed: int | None = None) -> None:
    """``ai.Train(model, dataset, TrainConfig(cuda=True, optimizer=...))``
    (crates/mmn-py/src/train/mod.rs:14-44): trains ``model`` for
    ``config.epochs`` epochs over ``dataset`` (any sized sequence of samples
    that ``model.backward`` understands), stepping the optimizer on the GPU."""
    samples = list(dataset)
    params = list(model.parameters())
    train_loop(config, list(model.param_order()), params,
               lambda i: model.backward(samples[i]), len(samples), seed=seed)
