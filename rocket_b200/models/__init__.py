from .moe_lm import MoELM
from .reference import ReferenceModel
from .weights import init_fuel_tensors

__all__ = ["MoELM", "ReferenceModel", "init_fuel_tensors"]
