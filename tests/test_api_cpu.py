"""Host-side API behaviour that needs no GPU: validation errors with the
reference's message fragments, policy helpers, surrogate registry, and the
no-CPU-fallback rule."""

from __future__ import annotations

import pytest
import torch

import myelin_b200 as mb
from myelin_b200 import checkpointing, surrogates


def test_checkpoint_policy_values_match_reference():
    # tests/test_checkpointing.py:12-15 of the reference
    assert checkpointing.recommended_checkpoint_size(100, policy="memory") == 10
    assert checkpointing.recommended_checkpoint_size(100, policy="balanced") == 25
    assert checkpointing.recommended_checkpoint_size(100, policy="speed") == 50
    assert checkpointing.resolve_checkpoint_size(256, "memory") == 16
    assert checkpointing.resolve_checkpoint_size(10, 25) == 10
    assert checkpointing.parse_checkpoint_size("speed") == "speed"
    assert checkpointing.parse_checkpoint_size("7") == 7
    for bad in (0, -3):
        with pytest.raises(ValueError, match="positive"):
            checkpointing.resolve_checkpoint_size(10, bad)
    with pytest.raises(ValueError, match="positive integer"):
        checkpointing.parse_checkpoint_size("fast")


def test_surrogate_registry_round_trips():
    for index, name in enumerate(surrogates.SURROGATE_NAMES):
        fn = surrogates.surrogate_from_name(name)
        assert surrogates.surrogate_name(fn) == name
        assert surrogates.surrogate_id(name) == index
    with pytest.raises(ValueError, match="built-in"):
        surrogates.surrogate_name(lambda c: c)


@pytest.mark.parametrize("name", surrogates.SURROGATE_NAMES)
def test_closed_form_derivative_matches_autograd_of_primitive(name):
    c = torch.linspace(-3.0, 3.0, 241, dtype=torch.float64).requires_grad_(True)
    c = c[(c.detach().abs() - 1.0).abs() > 1e-9].detach().requires_grad_(True)
    fn = surrogates.surrogate_from_name(name)
    (grad,) = torch.autograd.grad(fn(c).sum(), c)
    torch.testing.assert_close(surrogates.surrogate_derivative(c.detach(), name), grad,
                               rtol=1e-9, atol=1e-12)


def test_params_decay_properties():
    assert mb.LIFParams(tau_mem=10.0).decay == 1.0 - 1.0 / 10.0
    assert mb.ALIFParams(tau_adaptation=50.0).adaptation_decay == 1.0 - 1.0 / 50.0
    with pytest.raises(ValueError, match="positive"):
        _ = mb.LIFParams(tau_mem=0.0).decay


def test_scan_validation_messages_on_cpu():
    params = mb.LIFParams()
    with pytest.raises(ValueError, match=r"\[T, B, N\]"):
        mb.lif_forward(torch.zeros((2, 3)), mb.LIFState(torch.zeros((3,))), params)
    with pytest.raises(ValueError, match="must match inputs.shape"):
        mb.lif_forward(torch.zeros((2, 3, 4)), mb.LIFState(torch.zeros((3, 5))), params)
    with pytest.raises(ValueError, match="CUDA"):
        mb.lif_forward(torch.zeros((2, 3, 4)), mb.LIFState(torch.zeros((3, 4))), params)
    with pytest.raises(ValueError, match="unsupported backend"):
        mb.lif_forward(torch.zeros((2, 3, 4)), mb.LIFState(torch.zeros((3, 4))), params,
                       backend="numpy")  # type: ignore[arg-type]
    with pytest.raises(ValueError, match="hard_forward=True"):
        mb.surrogate_lif_forward(torch.zeros((2, 3, 4)), mb.LIFState(torch.zeros((3, 4))), params,
                                 hard_forward=False)
    with pytest.raises(ValueError, match="reset_mode"):
        mb.alif_forward(torch.zeros((2, 3, 4)),
                        mb.ALIFState(torch.zeros((3, 4)), torch.zeros((3, 4))),
                        mb.ALIFParams(), reset_mode="soft")  # type: ignore[arg-type]
    with pytest.raises(ValueError, match="unknown surrogate"):
        mb.surrogate_lif_forward(torch.zeros((2, 3, 4)), mb.LIFState(torch.zeros((3, 4))), params,
                                 surrogate="relu")  # type: ignore[arg-type]


def test_linear_validation_messages_on_cpu():
    params = mb.LIFParams()
    with pytest.raises(ValueError, match=r"\[T, B, F\]"):
        mb.linear_surrogate_lif_forward(torch.zeros((2, 3)), torch.zeros((3, 4)), None, params)
    with pytest.raises(ValueError, match="weight.shape"):
        mb.linear_surrogate_lif_forward(torch.zeros((2, 3, 5)), torch.zeros((3, 4)), None, params)
    with pytest.raises(ValueError, match="reduction"):
        mb.linear_surrogate_lif_rate_forward(torch.zeros((2, 3, 3)), torch.zeros((3, 4)), None,
                                             params, reduction="sum")  # type: ignore[arg-type]
    with pytest.raises(ValueError, match="positive"):
        mb.linear_surrogate_lif_rate_forward(torch.zeros((2, 3, 3)), torch.zeros((3, 4)), None,
                                             params, checkpoint_size=0)


def test_packing_validation_messages_on_cpu():
    with pytest.raises(ValueError, match="at least one dimension"):
        mb.pack_spikes(torch.tensor(1.0))
    with pytest.raises(ValueError, match="empty last dimension"):
        mb.pack_spikes(torch.empty((2, 0)))
    with pytest.raises(ValueError, match="CUDA"):
        mb.pack_spikes(torch.zeros((2, 5)))
    bad = mb.PackedSpikes(data=torch.zeros((2, 2), dtype=torch.int32), original_shape=(2, 65))
    with pytest.raises(ValueError, match="shape"):
        mb.unpack_spikes(bad)
    empty = mb.PackedSpikes(data=torch.zeros((2, 0), dtype=torch.int32), original_shape=(2, 0))
    with pytest.raises(ValueError, match="non-empty last dimension"):
        mb.packed_spike_count(empty)
    ok = mb.PackedSpikes(data=torch.zeros((3, 2, 2), dtype=torch.int32), original_shape=(3, 2, 35))
    with pytest.raises(ValueError, match="last dimension"):
        mb.packed_spike_counts(ok, dim=0)
    with pytest.raises(ValueError, match="duplicate"):
        mb.packed_spike_count(ok, dim=(0, -3))
    with pytest.raises(IndexError, match="out of range"):
        mb.packed_spike_count(ok, dim=5)


def test_packing_metadata_helpers():
    assert mb.packed_last_dim_size(0) == 0
    assert mb.packed_last_dim_size(33) == 2
    spikes = torch.zeros((100, 64, 2048))
    packed = mb.PackedSpikes(data=torch.zeros((100, 64, 64), dtype=torch.int32),
                             original_shape=(100, 64, 2048))
    assert mb.dense_spike_bytes(spikes) == 100 * 64 * 2048 * 4
    assert mb.packed_spike_bytes(packed) == 100 * 64 * 64 * 4
    assert mb.spike_compression_ratio(spikes, packed) == 32.0
    assert packed.original_numel == 100 * 64 * 2048


def test_modules_construct_with_reference_signatures():
    layer = mb.LinearSurrogateLIF(784, 1024, mb.LIFParams(tau_mem=20.0),
                                  surrogate=mb.fast_sigmoid_surrogate, surrogate_slope=25.0,
                                  stream_synapse=True, checkpoint_size="memory")
    assert layer.synapse.weight.shape == (784, 1024)
    assert layer.synapse.bias.shape == (1024,)
    rate = mb.LinearSurrogateLIFRate(4096, 10, surrogate=mb.superspike_surrogate,
                                     surrogate_slope=10.0, reduction="none")
    assert rate.reduction == "none" and rate.checkpoint_size == 25
    clf = mb.RateReadoutClassifier(784, 128, 10)
    assert clf.hidden.stream_synapse
    packed = mb.LinearSurrogateLIFPacked(10, 40)
    assert packed.synapse.weight.shape == (10, 40)
