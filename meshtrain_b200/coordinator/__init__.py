"""Control plane: worker registry, job planning, run artefacts and the HTTP API."""
