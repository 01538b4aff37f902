"""Model families: configs, synthetic weights, the f32 reference forward and the engine forward."""
