"""g2ptq_b200 -- B200-native (sm_100a) kernels for G2PTQ's per-layer
quantization hot path, behind the reference's quantizer-object API.

    from g2ptq_b200.gptq_utils.gptq_utils import GPTQ
    from g2ptq_b200.gptq_utils.g2ptq_utils import G2PTQ
    from g2ptq_b200.gptq_utils.gptaq_utils import GPTAQ
    from g2ptq_b200.gptq_utils.gptq_guided_utils import GPTQGuided
    from g2ptq_b200.utils.quant_utils import WeightQuantizer

The compute lives in ``_lib/libg2ptq_b200.so`` (C ABI: include/g2ptq_b200.h).
"""

__version__ = "0.1.0"
