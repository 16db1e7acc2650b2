"""Training steps replayed from a CUDA graph against the same steps run eagerly."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
           vocab_size=2048, intermediate_size=256, shared_intermediate_size=512, num_experts=4,
           top_k=2, routing_strategy="token_id_multi_hash", max_position_embeddings=256)


def _trainer(model, graph: bool):
    from complexity_framework_b200.training import Trainer, TrainingConfig

    cfg = TrainingConfig(learning_rate=2e-3, warmup_steps=4, lr_scheduler="cosine",
                         max_steps=12, precision="bf16", grad_clip=1.0,
                         distributed_mode="none", skip_param_update_check=True,
                         cuda_graph=graph, cuda_graph_warmup=2)
    return Trainer(model, cfg)


def test_graphed_steps_match_eager():
    from complexity_framework_b200 import ComplexityModel, ModelConfig

    torch.manual_seed(0)
    base = ComplexityModel(ModelConfig(**CFG)).cuda().to(torch.bfloat16)
    m_eager, m_graph = copy.deepcopy(base), copy.deepcopy(base)
    t_eager, t_graph = _trainer(m_eager, False), _trainer(m_graph, True)
    g = torch.Generator().manual_seed(1)
    # two batches repeated: the model can memorise them, so the loss must fall
    pair = [torch.randint(0, CFG["vocab_size"], (4, 128), generator=g).pin_memory()
            for _ in range(2)]
    batches = [pair[i % 2] for i in range(10)]
    le = [t_eager.train_step(b) for b in batches]
    lg = [t_graph.train_step(b) for b in batches]
    assert t_graph._graphed.graph is not None  # steps 3.. were replays
    assert t_graph.global_step == t_eager.global_step == 10
    assert t_graph.optimizer._step_count == t_eager.optimizer._step_count == 10
    # learning rate follows the schedule through the replays
    assert abs(t_graph.optimizer.param_groups[0]["lr"]
               - t_eager.optimizer.param_groups[0]["lr"]) < 1e-12
    for a, b in zip(le, lg):
        assert abs(a - b) < 2e-2 * max(1.0, abs(a)), (le, lg)
    assert le[-1] < le[0]
    for pa, pb in zip(m_eager.parameters(), m_graph.parameters()):
        assert float((pa.float() - pb.float()).abs().max()) < 5e-2
