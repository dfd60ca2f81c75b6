"""The trainer's optimizer loop (magicmindnet_b200/train.py, the Python mirror of
crates/mmn-train/src/lib.rs:354-448 and of ai.Train, crates/mmn-py/src/train/mod.rs:14-44).

CPU: the loop on an oracle stepper against a literal restatement of
train_with_encoder on the oracle (per-call ids, GradAccumulator averaging,
flushes with a ragged last batch): bit for bit. GPU: the GPU loop against the
oracle replay on the Chatbot(vocab 512, 2 layers, d_model 64) tensors over two
epochs: AdamW tensors bit for bit, Muon tensors within 2e-2 relative
Frobenius of their total update."""
import numpy as np
import pytest

from conftest import chatbot_params, rel_fro

N_SAMPLES = 10  # batch_size 3: batches of 3, 3, 3 and a ragged 1


def _grads(shapes, sample):
    rng = np.random.default_rng(1000 + sample)
    return [rng.normal(0, 1e-3, s).astype(np.float32) for s in shapes]


def _order(epoch):
    rng = np.random.default_rng(42 + epoch)
    idx = list(range(N_SAMPLES))
    for i in range(N_SAMPLES):
        j = int(rng.integers(0, N_SAMPLES))
        idx[i], idx[j] = idx[j], idx[i]
    return idx


class OracleStep:
    """One training step's per-call optimizer calls on the oracle: every tensor in
    call order with a new id, through HybridOptimizer.step or the trainer's
    separate AdamW (lib.rs:367-378), on GradAccumulator's averaged grads."""

    def __init__(self, oracle, config):
        R = oracle
        self.R = R
        self.use_hybrid = config.optimizer == "hybrid"
        self.hybrid = R.HybridOptimizer(R.MuonConfig(), R.AdamWConfig(lr=config.learning_rate),
                                        order=R.GEMM_F64)
        self.adamw = R.AdamW(R.AdamWConfig(lr=config.learning_rate))
        self.param_id = 0

    def step_host(self, grads, params, divisor):
        for g, p in zip(grads, params):
            avg = np.empty_like(g)
            self.R.lib().ref_grad_average(self.R._ptr(g), self.R._ptr(avg), g.size, int(divisor))
            if self.use_hybrid:
                self.hybrid.step(self.param_id, p, avg)
            else:
                self.adamw.step_param(self.param_id, p, avg)
            self.param_id += 1


def _literal(oracle, config, params, shapes):
    """train_with_encoder (lib.rs:382-442) written out on the oracle."""
    R = oracle
    hybrid = R.HybridOptimizer(R.MuonConfig(), R.AdamWConfig(lr=config.learning_rate),
                               order=R.GEMM_F64)
    adamw = R.AdamW(R.AdamWConfig(lr=config.learning_rate))
    use_hybrid = config.optimizer == "hybrid"
    param_id = 0

    def optim_step_weight(p, g):  # crates/mmn-models/src/chatbot.rs:208-227
        nonlocal param_id
        if use_hybrid:
            hybrid.step(param_id, p, g)
        else:
            adamw.step_param(param_id, p, g)
        param_id += 1

    batch_size = max(config.batch_size, 1)
    for epoch in range(config.epochs):
        idx = _order(epoch)
        accum = R.GradAccumulator()
        micro = 0
        for i, s in enumerate(idx):
            grads = _grads(shapes, s)
            if batch_size == 1:
                for p, g in zip(params, grads):
                    optim_step_weight(p, g)
                continue
            micro += 1
            accum.begin_micro_batch()
            for g in grads:
                accum.add_param_grad(g)
            accum.finish_micro_batch()
            if micro >= batch_size or i + 1 == len(idx):
                for k, p in enumerate(params):
                    optim_step_weight(p, accum.averaged_grad(k))
                accum.clear()
                micro = 0
    return param_id


def _model():
    rng = np.random.default_rng(0)
    named = chatbot_params(rng)
    return [n for n, _ in named], [v.shape for _, v in named], [v for _, v in named]


@pytest.mark.parametrize("optimizer,batch_size", [("hybrid", 3), ("adamw", 3), ("hybrid", 1)])
def test_loop_matches_literal_restatement(oracle, optimizer, batch_size):
    from magicmindnet_b200.step import TrainConfig
    from magicmindnet_b200.train import TrainLoop

    cfg = TrainConfig(epochs=2, batch_size=batch_size, cuda=True, optimizer=optimizer,
                      learning_rate=1e-3)
    _, shapes, p0 = _model()
    lit = [p.copy() for p in p0]
    lit_ids = _literal(oracle, cfg, lit, shapes)
    got = [p.copy() for p in p0]
    loop = TrainLoop(cfg, OracleStep(oracle, cfg), shapes)
    loop.run(N_SAMPLES, _order, lambda s: _grads(shapes, s), got)
    per_epoch = N_SAMPLES if batch_size == 1 else -(-N_SAMPLES // batch_size)
    assert loop.steps == 2 * per_epoch
    assert loop.param_id == lit_ids == 2 * per_epoch * len(shapes)
    for a, b in zip(got, lit):
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


def test_cpu_configuration_is_refused():
    from magicmindnet_b200.step import TrainConfig
    from magicmindnet_b200.train import train_loop

    with pytest.raises(ValueError, match="cuda=False"):
        train_loop(TrainConfig(cuda=False), [("w", (2, 2))], [np.zeros((2, 2), np.float32)],
                   lambda s: [np.zeros((2, 2), np.float32)], 1)


@pytest.mark.gpu
@pytest.mark.parametrize("optimizer,batch_size", [("hybrid", 3), ("hybrid", 1), ("muon", 3)])
def test_gpu_loop_matches_oracle_replay(mmn, oracle, optimizer, batch_size):
    from magicmindnet_b200.step import TrainConfig
    from magicmindnet_b200.train import TrainLoop, train_loop

    cfg = TrainConfig(epochs=2, batch_size=batch_size, cuda=True, optimizer=optimizer,
                      learning_rate=1e-3)
    names, shapes, p0 = _model()
    gpu = [p.copy() for p in p0]
    run = train_loop(cfg, list(zip(names, shapes)), gpu, lambda s: _grads(shapes, s), N_SAMPLES,
                     order=_order)
    ref = [p.copy() for p in p0]
    loop = TrainLoop(cfg, OracleStep(oracle, cfg), shapes)
    loop.run(N_SAMPLES, _order, lambda s: _grads(shapes, s), ref)
    assert run.steps == loop.steps and run.param_id == loop.param_id
    hybrid = optimizer == "hybrid"
    n_adamw = 0
    for n, s, a, b, p in zip(names, shapes, gpu, ref, p0):
        if hybrid and oracle.classify_param(s) == oracle.MATRIX:
            assert rel_fro(a - p, b - p) <= 2e-2, n
        else:
            n_adamw += 1
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32), err_msg=n)
    assert run.adamw_step == n_adamw * run.steps


@pytest.mark.gpu
def test_train_surface_runs_a_model(mmn, oracle):
    """Train(model, dataset, TrainConfig(cuda=True)) on a model object whose
    backward returns seeded grads per sample: the same weights as the loop."""
    from magicmindnet_b200.step import TrainConfig
    from magicmindnet_b200.train import Train, TrainLoop

    names, shapes, p0 = _model()

    class Model:
        def __init__(self):
            self.weights = [p.copy() for p in p0]

        def param_order(self):
            return list(zip(names, shapes))

        def parameters(self):
            return self.weights

        def backward(self, sample):
            return _grads(shapes, sample)

    cfg = TrainConfig(epochs=1, batch_size=4, cuda=True, optimizer="hybrid", learning_rate=1e-3)
    model = Model()
    Train(model, list(range(N_SAMPLES)), cfg, seed=7)
    # the same shuffle, replayed on the oracle
    rng = np.random.default_rng(7)

    def order(_epoch):
        idx = list(range(N_SAMPLES))
        for i in range(N_SAMPLES):
            j = int(rng.integers(0, N_SAMPLES))
            idx[i], idx[j] = idx[j], idx[i]
        return idx

    ref = [p.copy() for p in p0]
    TrainLoop(cfg, OracleStep(oracle, cfg), shapes).run(N_SAMPLES, order,
                                                          lambda s: _grads(shapes, s), ref)
    for n, s, a, b, p in zip(names, shapes, model.weights, ref, p0):
        if oracle.classify_param(s) == oracle.MATRIX:
            assert rel_fro(a - p, b - p) <= 2e-2, n
        else:
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32), err_msg=n)
