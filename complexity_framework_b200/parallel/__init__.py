"""Parallel runtime: process groups, data/tensor/pipeline/expert parallelism, 3-D layout."""
from .cluster import ClusterConfig, ClusterModel, ProcessGroupManager
from .data_parallel import (GradientAccumulator, PrecisionMode, ShardingMode,
                            broadcast_parameters, simple_ddp, wrap_model_fsdp)
from .distributed import (barrier, cleanup_distributed, configure_nccl, dist_timeout_s,
                          get_rank, get_world_size, init_distributed, is_main_process, safe_main)
from .expert_parallel import ExpertParallelRouted, all_to_all, make_expert_parallel
from .pipeline_parallel import (PipelineModel, PipelineScheduler, PipelineStage,
                                split_model_for_pipeline)
from .tensor_parallel import (ColumnParallelLinear, ParallelEmbedding, RowParallelLinear,
                              copy_to_tp, gather_from_tp, gather_tp_state_dict, get_tp_group,
                              initialize_tensor_parallel, make_parallel, reduce_from_tp,
                              scatter_to_tp)
