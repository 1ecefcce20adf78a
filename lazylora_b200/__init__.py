"""
lazylora_b200: the routed-expert MXFP4 path of LazyLoRA (heyobi/LazyLora) on NVIDIA B200.

Entry points mirroring the reference's:
  lazylora_b200.native.kernel()                 -> lazy_lora.native.kernel()   (gemm / gemm_t / dequant)
  lazylora_b200.core.moe_router.KimiK3MoERouter -> lazy_lora.core.moe_router.KimiK3MoERouter
  lazylora_b200.trainer.routed_experts          -> RoutedExpertsFunction and the expert sweep of
                                                   lazy_lora.trainer.lazy_trainer.LazyLoRATrainer
The CUDA library (liblazylora_b200.so, C ABI in include/lazylora_b200.h) is built in-tree by
`python -m lazylora_b200.build`.
"""
__version__ = "0.1.0"
