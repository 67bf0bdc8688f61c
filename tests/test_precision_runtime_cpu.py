"""Precision runtime on CPU: dynamic loss scaling (scale, unscale, skip on overflow, back-off, growth),
optimizer-owned master weights for persistent low-bit layers and their shard domains, and the ZeRO
optimizer's state dtypes and partitioning rule.

Behaviour follows the reference's tests test_runtime_mixed_precision.py, test_master_store_binding.py,
test_zero_external_master_mapping.py, test_zero_optimizer_dtype_split.py and test_zero_partitioning.py."""
import argparse

import pytest
import torch
import torch.nn as nn

from nano_train_b200.distributed.zero import DistributedOptimizerConfig, MegatronZeroOptimizer, _compute_shard
from nano_train_b200.layers import Linear
from nano_train_b200.parallel.sync import collect_param_shard_info
from nano_train_b200.precision.master_store import get_lowbit_master_store, materialize_optimizer_owned_masters
from nano_train_b200.precision.mixed_precision import (MixedPrecisionController, build_module_precision_resolver,
                                                       resolve_precision_config)

CPU = torch.device("cpu")


def _config(**flags):
    return resolve_precision_config(argparse.Namespace(**flags), CPU)


def test_cpu_defaults_to_fp32_without_loss_scaling():
    cfg = _config()
    assert cfg.mode == "fp32" and cfg.activation_dtype == "fp32" and cfg.params_dtype == "fp32"
    ctl = MixedPrecisionController(cfg, device=CPU)
    assert not ctl.uses_loss_scaling


def _fp8_controller(**kw):
    return MixedPrecisionController(_config(fp8=True, fp8_backend="emulated", **kw), device=CPU)


def test_loss_is_scaled_gradients_unscaled_and_overflow_backs_off():
    ctl = _fp8_controller(loss_scale_init=1024.0, loss_scale_min=64.0)
    assert ctl.uses_loss_scaling
    w = nn.Parameter(torch.tensor([2.0, -1.0]))
    m = nn.Module()
    m.w = w
    ctl.backward((w * torch.tensor([3.0, 5.0])).sum())
    torch.testing.assert_close(w.grad, torch.tensor([3.0, 5.0]) * 1024)
    assert ctl.prepare_optimizer_step(m)
    torch.testing.assert_close(w.grad, torch.tensor([3.0, 5.0]))
    ctl.update_after_step(step_applied=True)
    assert ctl.runtime_state.loss_scale == 1024.0

    for expected in (512.0, 256.0, 128.0, 64.0, 64.0):  # x0.5 per overflow, clamped at the minimum
        w.grad = torch.tensor([float("inf"), 1.0])
        assert not ctl.prepare_optimizer_step(m)
        ctl.update_after_step(step_applied=False)
        assert ctl.runtime_state.loss_scale == expected
    assert ctl.runtime_state.skipped_steps == 5 and ctl.runtime_state.found_inf_steps == 5
    w.grad = torch.tensor([float("nan"), 0.0])
    assert not ctl.prepare_optimizer_step(m)


def test_loss_scale_grows_after_the_interval_and_is_capped():
    ctl = _fp8_controller(loss_scale_init=8.0, loss_scale_growth_interval=3, loss_scale_max=32.0)
    scales = []
    for _ in range(12):
        ctl.update_after_step(step_applied=True)
        scales.append(ctl.runtime_state.loss_scale)
    assert scales == [8, 8, 16, 16, 16, 32, 32, 32, 32, 32, 32, 32]
    ctl.update_after_step(step_applied=True)
    ctl.update_after_step(step_applied=False)  # an overflow resets the growth counter
    assert ctl.runtime_state.growth_tracker == 0 and ctl.runtime_state.loss_scale == 16.0


@pytest.mark.parametrize("flags, message", [
    (dict(loss_scale_init=0.0), "loss-scale-init"), (dict(loss_scale_growth_factor=1.0), "growth-factor"),
    (dict(loss_scale_backoff_factor=1.0), "backoff-factor"), (dict(loss_scale_growth_interval=0), "interval"),
    (dict(loss_scale_min=8.0, loss_scale_max=4.0), "loss-scale-max"), (dict(fp8_format="e5m2"), "fp8-format")])
def test_loss_scale_and_format_flags_are_validated(flags, message):
    with pytest.raises(ValueError, match=message):
        _config(fp8=True, fp8_backend="emulated", **flags)


class _Net(nn.Module):
    def __init__(self, resolver):
        super().__init__()
        self.fc = Linear(16, 16, module_path="fc", precision_resolver=resolver)
        self.head = Linear(16, 4, module_path="head", precision_resolver=resolver)

    def forward(self, x):
        return self.head(torch.relu(self.fc(x)))


def test_optimizer_owned_masters_rebind_the_module_weight_and_train():
    torch.manual_seed(0)
    cfg = _config(fp8_param=True, persistent_lowbit_include=["^fc$"], lowbit_master_ownership="optimizer")
    net = _Net(build_module_precision_resolver(cfg))
    w_before = net.fc.weight.detach().clone()
    store = materialize_optimizer_owned_masters(net, precision_config=cfg)
    assert store is get_lowbit_master_store(net) and list(store.masters.keys()) == ["fc__weight"]
    meta = store.metadata["fc__weight"]
    assert (meta.module_path, meta.parameter_name, meta.shard_domain, meta.shape) == \
        ("fc", "weight", "data_parallel", (16, 16))
    assert net.fc.weight is store.masters["fc__weight"] and torch.equal(net.fc.weight, w_before)
    # the master is counted once among the model's parameters and receives the gradient
    assert sum(1 for p in net.parameters() if p is net.fc.weight) == 1
    opt = torch.optim.SGD(net.parameters(), lr=0.1)
    x, y = torch.randn(32, 16), torch.randn(32, 4)
    first = None
    for _ in range(10):
        opt.zero_grad()
        loss = nn.functional.mse_loss(net(x), y)
        loss.backward()
        assert net.fc.weight.grad is not None
        opt.step()
        net.fc.refresh_persistent_lowbit_params()
        first = loss.item() if first is None else first
    assert loss.item() < first


def test_master_store_is_skipped_for_module_ownership_and_follows_expert_domains():
    cfg = _config(fp8_param=True, lowbit_master_ownership="module")
    assert materialize_optimizer_owned_masters(_Net(build_module_precision_resolver(cfg)), precision_config=cfg) is None

    cfg = _config(fp8_param=True, lowbit_master_ownership="optimizer")
    r = build_module_precision_resolver(cfg)
    net = nn.Module()
    net.dense = Linear(8, 8, module_path="layers.0.mlp.fc", precision_resolver=r)
    net.expert = Linear(8, 8, module_path="layers.0.mlp.experts.3.fc1", precision_resolver=r)
    store = materialize_optimizer_owned_masters(net, precision_config=cfg)
    domains = {m.module_path: m.shard_domain for m in store.metadata.values()}
    assert domains == {"layers.0.mlp.fc": "data_parallel", "layers.0.mlp.experts.3.fc1": "expert_model_parallel"}
    info = collect_param_shard_info(net)
    assert info.expert_model_parallel_sharded_param_ids == {id(net.expert.weight)}
    assert info.tensor_model_parallel_sharded_param_ids == set()


def test_compute_shard_covers_without_overlap():
    for numel in (1, 7, 64, 1000, 1023):
        for size in (1, 2, 3, 4, 8):
            covered = []
            for r in range(size):
                s, e, chunk = _compute_shard(numel, r, size)
                assert chunk == -(-numel // size) and 0 <= s <= e <= numel and e - s <= chunk
                covered.extend(range(s, e))
            assert covered == list(range(numel))


def _zero(model, **dtypes):
    cfg = DistributedOptimizerConfig(use_distributed_optimizer=True, data_parallel_sharding_strategy="optim",
                                     **dtypes)
    return MegatronZeroOptimizer(model, cfg, None, None, set())


def test_state_uses_the_configured_dtypes_and_loads_into_them():
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(8, 8), nn.Linear(8, 3))
    opt = _zero(model, main_params_dtype="fp32", exp_avg_dtype="bf16", exp_avg_sq_dtype="fp16")
    for st in opt.state.values():
        assert (st["master_param"].dtype, st["exp_avg"].dtype, st["exp_avg_sq"].dtype) == \
            (torch.float32, torch.bfloat16, torch.float16)
    x = torch.randn(4, 8)
    for _ in range(2):
        opt.zero_grad()
        model(x).square().mean().backward()
        opt.step()
    saved = opt.get_parameter_state_dp_zero(include_tensors=True)
    assert saved["optimizer_state_dtypes"] == {"main_params_dtype": "fp32", "main_grads_dtype": "fp32",
                                               "exp_avg_dtype": "bf16", "exp_avg_sq_dtype": "fp16"}
    # fp32 tensors in the payload are cast into the existing low-precision state
    for rec in saved["parameters"].values():
        rec["exp_avg"] = rec["exp_avg"].float()
    opt2 = _zero(nn.Sequential(nn.Linear(8, 8), nn.Linear(8, 3)), exp_avg_dtype="bf16", exp_avg_sq_dtype="fp16")
    opt2.load_parameter_state_from_dp_zero(saved)
    for (n, a), b in zip(saved["parameters"].items(), opt2.state.values()):
        assert b["exp_avg"].dtype == torch.bfloat16 and torch.equal(b["exp_avg"].float(), a["exp_avg"])
        assert b["step"] == 2
    with pytest.raises(ValueError, match="Unsupported optimizer dtype alias"):
        _zero(model, exp_avg_dtype="fp8")


def test_signature_is_stable_for_the_same_architecture_and_sees_shape_and_expert_changes():
    mk = lambda h: nn.Sequential(nn.Linear(8, h), nn.Linear(h, 3))  # noqa: E731
    a, b = _zero(mk(8)), _zero(mk(8))
    assert a.parameter_signature_hash() == b.parameter_signature_hash()
    assert a.parameter_signature_hash() != _zero(mk(9)).parameter_signature_hash()
    m = mk(8)
    cfg = DistributedOptimizerConfig(use_distributed_optimizer=True, data_parallel_sharding_strategy="optim")
    expert = MegatronZeroOptimizer(m, cfg, None, None, {id(m[0].weight)})
    assert expert.parameter_signature_hash() != a.parameter_signature_hash()
    meta = expert._meta_by_name["0.weight"]
    assert meta.is_expert_param and (meta.shard_start, meta.shard_end, meta.group_size) == (0, 64, 1)


def _padamw(model, **dt):
    from nano_train_b200.runtime.optimizer_runtime import PrecisionAdamW

    d = dict(main_params_dtype="fp32", main_grads_dtype="fp32", exp_avg_dtype="fp32", exp_avg_sq_dtype="fp32")
    d.update(dt)
    return PrecisionAdamW(model.parameters(), lr=1e-2, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8, **d)


def test_precision_adamw_matches_torch_and_skips_parameters_without_gradients():
    torch.manual_seed(0)
    model, ref = nn.Sequential(nn.Linear(6, 5), nn.Linear(5, 3)), nn.Sequential(nn.Linear(6, 5), nn.Linear(5, 3))
    ref.load_state_dict(model.state_dict())
    opt = _padamw(model)
    ref_opt = torch.optim.AdamW(ref.parameters(), lr=1e-2, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8)
    x = torch.randn(8, 6)
    for step in range(4):
        for m, o in ((model, opt), (ref, ref_opt)):
            o.zero_grad()
            m(x).square().mean().backward()
            if step == 3:  # the first layer's bias gets no gradient: value and state stay as they are
                m[0].bias.grad = None
            o.step()
    for p, r in zip(model.parameters(), ref.parameters()):
        torch.testing.assert_close(p, r, atol=1e-6, rtol=1e-5)
    assert opt.state[model[0].bias]["step"] == 3 and opt.state[model[0].weight]["step"] == 4


def test_precision_adamw_state_dict_resumes_identically_with_low_precision_moments():
    torch.manual_seed(1)
    a = nn.Linear(7, 4)
    b = nn.Linear(7, 4)
    b.load_state_dict(a.state_dict())
    oa = _padamw(a, exp_avg_dtype="bf16", exp_avg_sq_dtype="bf16")
    assert oa.state[a.weight]["exp_avg"].dtype == torch.bfloat16
    x = torch.randn(5, 7)

    def step(m, o):
        o.zero_grad()
        m(x).square().mean().backward()
        o.step()

    step(a, oa)
    ob = _padamw(b, exp_avg_dtype="bf16", exp_avg_sq_dtype="bf16")
    ob.load_state_dict(oa.state_dict())
    b.load_state_dict(a.state_dict())
    step(a, oa)
    step(b, ob)
    assert torch.equal(a.weight, b.weight) and torch.equal(a.bias, b.bias)
    with pytest.raises(ValueError, match="not a PrecisionAdamW"):
        ob.load_state_dict({"format": "other"})
    with pytest.raises(ValueError, match="parameter layout"):
        _padamw(nn.Linear(7, 5)).load_state_dict(oa.state_dict())


def test_step_with_sync_policy_syncs_then_steps_or_uses_ready_grads():
    from types import SimpleNamespace

    from nano_train_b200.runtime.contracts import OptimizerState, ParamShardInfo
    from nano_train_b200.runtime.optimizer_runtime import step_with_sync_policy, zero_grad_optimizer

    calls = []

    class Opt:
        def zero_grad(self, set_to_none=True):
            calls.append(("zero_grad", set_to_none))

        def step(self):
            calls.append(("step",))

        def step_with_ready_grads(self):
            calls.append(("ready",))

    parallel = SimpleNamespace(data_parallel_size=2, expert_data_parallel_size=2, data_parallel_group="dp",
                               expert_data_parallel_group="edp")
    state = OptimizerState(optimizer=Opt(), shard_info=ParamShardInfo(set(), set()))

    def sync(**kw):
        calls.append(("sync", kw["data_parallel_group"], kw["expert_data_parallel_group"]))

    zero_grad_optimizer(state)
    ctx = SimpleNamespace(parallel=parallel, run_config=SimpleNamespace(args=SimpleNamespace(
        use_distributed_optimizer=False)))
    step_with_sync_policy(model=nn.Linear(1, 1), state=state, ctx=ctx, synchronize_gradients_fn=sync)
    ctx.run_config.args.use_distributed_optimizer = True
    step_with_sync_policy(model=nn.Linear(1, 1), state=state, ctx=ctx, synchronize_gradients_fn=sync)
    assert calls == [("zero_grad", True), ("sync", "dp", "edp"), ("step",), ("ready",)]
    with pytest.raises(TypeError, match="step_with_ready_grads"):
        step_with_sync_policy(model=nn.Linear(1, 1), state=OptimizerState(optimizer=object(), shard_info=None),
                              ctx=ctx, synchronize_gradients_fn=sync)
