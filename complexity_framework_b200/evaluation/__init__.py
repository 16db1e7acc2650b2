"""Evaluation: perplexity and text metrics, multiple-choice benchmarks,
synthetic recall probes."""
from .benchmarks import (ARCBenchmark, BENCHMARKS, BenchmarkResult, BenchmarkRunner,
                         HellaSwagBenchmark, MMLUBenchmark, PIQABenchmark, TruthfulQABenchmark,
                         WinograndeBenchmark, choice_logprobs)
from .metrics import (BertScoreEvaluator, bleu, distinct_n, self_bleu, compute_accuracy, compute_f1, compute_perplexity,
                      exact_match, expected_calibration_error, perplexity_from_loss, rouge,
                      token_f1)
from .recall import (RecallBatch, RecallMetrics, build_associative_recall_batch,
                     build_induction_batch, score_target_logits)
