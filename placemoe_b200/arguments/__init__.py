from .parser import Arguments, DataArguments, HierMoEConfig, ModelArguments, TrainingArguments, parse_args, save_args

__all__ = ["Arguments", "DataArguments", "HierMoEConfig", "ModelArguments", "TrainingArguments", "parse_args",
           "save_args"]
