"""myelin_b200: B200-native (sm_100a) kernels for the spiking-network hot path of myelin.

Public names mirror ``myelin``'s for the LIF/ALIF scan, the stream-synapse
modules, bit-packed spikes and their collectives. All compute runs in the
hand-written CUDA library ``libmyelin_b200.so`` (see ``include/myelin_b200.h``).
"""

from myelin_b200.checkpointing import (
    CheckpointPolicy,
    CheckpointSize,
    parse_checkpoint_size,
    recommended_checkpoint_size,
    resolve_checkpoint_size,
)
from myelin_b200.distributed import (
    distributed_available_and_initialized,
    packed_spike_all_gather,
    packed_spike_all_gather_into_tensor,
    PackedSpikeExchange,
    packed_spike_count_all_reduce,
    packed_spike_rate_all_reduce,
)
from myelin_b200.kernels import (
    Backend,
    alif_forward,
    izhikevich_forward,
    izhikevich_step,
    fused_lif_unroll,
    lif_forward,
    lif_forward_packed_spikes,
    linear_surrogate_lif_forward,
    linear_surrogate_lif_packed_forward,
    two_layer_surrogate_lif_rate_packed_hidden_forward,
    two_layer_surrogate_lif_rate_recompute_forward,
    linear_surrogate_lif_rate_forward,
    surrogate_alif_forward,
    surrogate_lif_forward,
)
from myelin_b200.modules import (
    ALIFCell,
    IzhikevichCell,
    LIFCell,
    LinearLIF,
    LinearSurrogateLIF,
    LinearSurrogateLIFPacked,
    LinearSurrogateLIFRate,
    LinearSynapse,
    RateReadoutClassifier,
    SurrogateALIFCell,
    SurrogateLIFCell,
    TimeUnroll,
)
from myelin_b200.neurons import (
    ALIFParams,
    ALIFState,
    IzhikevichParams,
    IzhikevichState,
    LIFParams,
    LIFState,
)
from myelin_b200.packing import (
    BITS_PER_WORD,
    PackedSpikes,
    dense_spike_bytes,
    pack_spikes,
    packed_last_dim_size,
    packed_spike_bytes,
    packed_spike_count,
    packed_spike_counts,
    packed_spike_counts_over_leading_dims,
    pack_spikes_with_counts,
    packed_spike_rate,
    spike_compression_ratio,
    unpack_spikes,
)
from myelin_b200.surrogates import (
    SURROGATE_NAMES,
    SurrogateName,
    atan_surrogate,
    fast_sigmoid_surrogate,
    hard_surrogate_spike,
    multi_gaussian_surrogate,
    sigmoid_surrogate,
    superspike_surrogate,
    surrogate_derivative,
    surrogate_from_name,
    surrogate_name,
    triangular_surrogate,
)

__version__ = "0.1.0"
