"""Build bookkeeping of libvgb200 (CPU): objects compiled with other knob defines are never reused."""

import os

from voronoi_gauss_b200 import build


def _touch(path):
    with open(path, 'w') as f:
        f.write('x')


def test_changed_defines_invalidate_objects(tmp_path):
    obj_dir = str(tmp_path)
    build._sync_flags(obj_dir, ('VG_FWD_PREFETCH=1',))
    _touch(os.path.join(obj_dir, 'foam.o'))
    # same knobs: the object stays
    build._sync_flags(obj_dir, ('VG_FWD_PREFETCH=1',))
    assert os.path.exists(os.path.join(obj_dir, 'foam.o'))
    # other knobs (or none): the object goes and the new signature is recorded
    build._sync_flags(obj_dir, ())
    assert not os.path.exists(os.path.join(obj_dir, 'foam.o'))
    with open(os.path.join(obj_dir, 'flags.txt')) as f:
        assert f.read() == build.flag_signature(())


def test_signature_ignores_define_order():
    assert build.flag_signature(('A=1', 'B=2')) == build.flag_signature(('B=2', 'A=1'))
    assert build.flag_signature(('A=1',)) != build.flag_signature(('A=2',))
