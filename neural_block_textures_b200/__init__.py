"""neural_block_textures_b200: a B200 (sm_100a) Evolution Strategies training backend for
neural_block_textures, behind the reference's ntc_cuda::Trainer interface.

The product is libntc_b200.so (CUDA kernels + host engine + C ABI + the C++ class). This package
builds it (build.py), binds it (abi.py, trainer.py) and describes models and benchmark
configurations (model.py, synth.py, dct.py).
"""
from .abi import DctDesc, ModelDesc, QesDesc, load_library
from .model import CONFIGS, LevelSpec, ModelSpec, TrainConfig, config, qat_grid_table
from .trainer import Trainer

__all__ = ["Trainer", "ModelDesc", "QesDesc", "DctDesc", "load_library", "ModelSpec", "LevelSpec", "TrainConfig",
           "CONFIGS", "config", "qat_grid_table"]
