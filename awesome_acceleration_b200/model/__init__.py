"""Qwen3 model classes with the reference's module interface
(yijichar/AWesome_ACceleration model/model.py, model/model_tp.py,
model/parallel_layers.py, model/distributed.py) running on the B200 kernels."""
