"""Pipeline layer: DiffletPipeline, parallel config, artefact cache, TeaCache, bucketing."""
