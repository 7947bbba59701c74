"""B200-native DeformableFeatureAggregation (DFA) hot path of Sparse4D v3.

Public API:
  DeformableFeatureAggregation, preprocess_dfa_parameters   -- drop-in module (dfa.py)
  deformable_aggregation, kps_project, kps_project_fused,
  pack_feature_maps, level_tables, weights_fc_into,
  output_proj_into, camera_logits_into                      -- operators (ops.py)
  DFAStack, PipelinedDFAStack, capture                      -- CUDA-graph execution (graph.py)
  chained_camera_terms                                      -- next layer's camera terms beside this gather
  InstanceBank, project_anchors                             -- temporal instances (instance_bank.py)
  Sparse4DHead, HeadGraph, preprocess_head_parameters       -- the decoder chain around the DFA (head.py)
The operators run hand-written sm_100a CUDA kernels from lib/libs4d_dfa.so through the C ABI
of include/s4d_dfa.h; the library is loaded on first use and its absence raises.
"""
from . import synthetic  # noqa: F401
from .dfa import DeformableFeatureAggregation, preprocess_dfa_parameters  # noqa: F401
from .graph import DFAStack, PipelinedDFAStack, capture, chained_camera_terms  # noqa: F401
from .head import HeadGraph, Sparse4DHead, preprocess_head_parameters  # noqa: F401
from .instance_bank import InstanceBank, preprocess_instance_bank_parameters, project_anchors  # noqa: F401
from .ops import (  # noqa: F401
    deformable_aggregation,
    deformable_aggregation_into,
    kps_project,
    kps_project_fused,
    kps_project_into,
    camera_logits_into,
    level_tables,
    output_proj_into,
    pack_feature_maps,
    visible_indices,
    weights_fc_into,
)
