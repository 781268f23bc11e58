"""A reference user's config files load unchanged: every YAML the reference ships parses under this
package's schema and builds its model.  The reference tree is read from ``MESHTRAIN_REFERENCE_ROOT``
(default: the checkout this package was built against); the test skips where it is absent."""

import glob
import os

import pytest
import yaml

from meshtrain_b200.config import parse_config

ROOT = os.environ.get("MESHTRAIN_REFERENCE_ROOT", "/root/reference")
FILES = sorted(glob.glob(os.path.join(ROOT, "configs", "*.yaml")))


@pytest.mark.skipif(not FILES, reason="reference configs not available")
@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(p) for p in FILES])
def test_reference_config_parses_and_builds(path):
    with open(path) as f:
        cfg = parse_config(yaml.safe_load(f))
    spec = cfg.build_model_spec()
    assert spec.num_layers > 0 and cfg.training.num_microbatches >= 1
