"""Quantization: int8 / int4 / FP8 linear layers, dynamic + static quantizers,
GPTQ, AWQ and a GGUF writer."""
from .awq import AWQConfig, AWQLinear, AWQQuantizer, awq_quantize
from .gguf import GGUFQuantType, GGUFTensorInfo, GGUFWriter, export_gguf, read_gguf_header
from .gptq import GPTQConfig, GPTQSolver, gptq_quantize_model
from .quantizer import (DynamicQuantizer, Linear4bit, Linear8bit, LinearFP8, QuantizationConfig,
                        QuantizationMethod, StaticQuantizer, compare_outputs, get_model_size,
                        quantize_model)
