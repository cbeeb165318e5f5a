from .schema import (BoosterConfig, ConfigError, DeltaNetConfig, EngineConfig, FuelConfig,
                     ModelConfig, RocketConfig, load_booster, load_engine, load_fuel,
                     load_rocket, model_config)

__all__ = ["BoosterConfig", "ConfigError", "DeltaNetConfig", "EngineConfig", "FuelConfig",
           "ModelConfig", "RocketConfig", "load_booster", "load_engine", "load_fuel",
           "load_rocket", "model_config"]
