"""delta_block_lm_b200: the GDN-2 hot path of delta-block-lm, rebuilt for NVIDIA B200 (sm_100a).

The kernels live in ``libdbl_gdn2.so`` (C ABI: ``include/dbl_gdn2.h``); this package is the
host-side mirror of the reference's kernel and mixer entry points over torch CUDA tensors.
"""
from .kernels import (GdnTrainingGrads, GdnTrainingOutput, gdn2_decode_step, gdn2_prefill, gdn2_prefill_host,
                      gdn2_prefill_segmented, gdn2_prefill_time_sharded_devices, gdn2_prologue, gdn2_scan,
                      gdn2_scan_backward, gdn2_span_fold, gdn2_span_transition, gdn_training_backward,
                      gdn_training_backward_saved, gdn_training_scan, gdn_training_scan_saved)
from .mixers import MixerKind, ScanBackend, ScanInput, ScanOutput, scan_selected
from .relay import relay_attention_forward, relay_merge_decode, relay_workspace_bytes

__all__ = [
    "GdnTrainingOutput", "GdnTrainingGrads", "gdn_training_scan", "gdn_training_backward", "gdn_training_scan_saved",
    "gdn_training_backward_saved", "gdn2_prologue", "gdn2_scan", "gdn2_scan_backward", "gdn2_prefill", "gdn2_prefill_host", "gdn2_span_transition",
    "gdn2_span_fold", "gdn2_prefill_segmented", "gdn2_prefill_time_sharded_devices",
    "gdn2_decode_step", "relay_attention_forward", "relay_merge_decode", "relay_workspace_bytes", "MixerKind", "ScanBackend",
    "ScanInput", "ScanOutput", "scan_selected",
]
