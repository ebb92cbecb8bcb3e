from mint_b200.sft.peft.lora import LoRA, LoRALinear
from mint_b200.sft.peft.qlora import QLoRA, QLoRALinear

__all__ = ["LoRA", "LoRALinear", "QLoRA", "QLoRALinear"]
