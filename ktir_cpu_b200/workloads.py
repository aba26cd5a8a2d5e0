"""KTIR source generators for the five benchmark workloads, plus seeded inputs.

Each generator returns KTIR MLIR text written for this backend (none of these
kernels exist in the ktir-cpu examples).  They are ordinary KTIR: the NumPy
reference interpreter executes them unchanged, which is what makes it a
usable oracle, and every per-core live set stays inside the 2 MiB LX
scratchpad that interpreter enforces.

  vector_add   1-D f16 add, one load/add/store per core
  softmax      row softmax, f32 max/sum reductions, f16 in/out, rows chunked
  gemm         C = A @ B, f16 operands widened to f32, f32 accumulation over a
               K loop of 128-wide tiles, one output block per core
  gather_add   indirect row gather -> +1.0 -> indirect row scatter
  attention    causal multi-head attention as an online-softmax loop over
               K/V blocks (the form the attention rewrite recognises)
"""

from __future__ import annotations

from typing import Dict, Tuple

import numpy as np


def _box(shape: Tuple[int, ...]) -> str:
    dims = ", ".join(f"d{i}" for i in range(len(shape)))
    cons = ", ".join(f"d{i} >= 0, -d{i} + {s - 1} >= 0" for i, s in enumerate(shape))
    return f"affine_set<({dims}) : ({cons})>"


def _ident(n: int) -> str:
    dims = ", ".join(f"d{i}" for i in range(n))
    return f"affine_map<({dims}) -> ({dims})>"


def _view(name: str, ptr: str, shape, dtype: str) -> str:
    strides = []
    acc = 1
    for s in reversed(shape):
        strides.append(acc)
        acc *= s
    strides = list(reversed(strides))
    ty = "x".join(str(s) for s in shape) + "x" + dtype
    return (f"    {name} = ktdp.construct_memory_view {ptr}, sizes: {list(shape)}, "
            f"strides: {strides} {{\n"
            f"      coordinate_set = {_box(tuple(shape))},\n"
            f"      memory_space = #ktdp.spyre_memory_space<HBM>\n"
            f"    }} : memref<{ty}>\n")


def _tile(name: str, view: str, idx, vshape, dtype: str, tshape) -> str:
    vty = "x".join(str(s) for s in vshape) + "x" + dtype
    tty = "x".join(str(s) for s in tshape)
    return (f"{name} = ktdp.construct_access_tile {view}[{', '.join(idx)}] {{\n"
            f"        access_tile_set = {_box(tuple(tshape))},\n"
            f"        access_tile_order = {_ident(len(tshape))}\n"
            f"      }} : memref<{vty}> -> !ktdp.access_tile<{tty}xindex>\n")


# ---------------------------------------------------------------------------

def vector_add(n: int = 1024, grid: int = 1) -> str:
    assert n % grid == 0
    blk = n // grid
    return f"""module {{
  func.func @add_kernel(%x_ptr: index, %y_ptr: index, %out_ptr: index) attributes {{grid = [{grid}]}} {{
    %core = ktdp.get_compute_tile_id : index
    %blk = arith.constant {blk} : index
    %off = arith.muli %core, %blk : index
{_view('%xv', '%x_ptr', (n,), 'f16')}{_view('%yv', '%y_ptr', (n,), 'f16')}{_view('%ov', '%out_ptr', (n,), 'f16')}
    {_tile('%xt', '%xv', ['%off'], (n,), 'f16', (blk,))}
    {_tile('%yt', '%yv', ['%off'], (n,), 'f16', (blk,))}
    %x = ktdp.load %xt : !ktdp.access_tile<{blk}xindex> -> tensor<{blk}xf16>
    %y = ktdp.load %yt : !ktdp.access_tile<{blk}xindex> -> tensor<{blk}xf16>
    %sum = arith.addf %x, %y : tensor<{blk}xf16>
    {_tile('%ot', '%ov', ['%off'], (n,), 'f16', (blk,))}
    ktdp.store %sum, %ot : tensor<{blk}xf16>, !ktdp.access_tile<{blk}xindex>
    return
  }}
}}
"""


def softmax(rows: int = 4096, cols: int = 1024, grid: int = 32, chunk: int = 32) -> str:
    assert rows % grid == 0
    per = rows // grid
    assert per % chunk == 0
    t = f"{chunk}x{cols}"
    bmaps = ("[affine_map<(d0, d1) -> (d0, d1)>, affine_map<(d0, d1) -> (d0)>, "
             "affine_map<(d0, d1) -> (d0, d1)>]")
    return f"""module {{
  func.func @softmax_rows(%in_ptr: index, %out_ptr: index) attributes {{grid = [{grid}]}} {{
    %core = ktdp.get_compute_tile_id : index
    %c0 = arith.constant 0 : index
    %per = arith.constant {per} : index
    %step = arith.constant {chunk} : index
    %row0 = arith.muli %core, %per : index
    %row1 = arith.addi %row0, %per : index
{_view('%iv', '%in_ptr', (rows, cols), 'f16')}{_view('%ov', '%out_ptr', (rows, cols), 'f16')}
    scf.for %r = %row0 to %row1 step %step {{
      {_tile('%it', '%iv', ['%r', '%c0'], (rows, cols), 'f16', (chunk, cols))}
      %x16 = ktdp.load %it : !ktdp.access_tile<{t}xindex> -> tensor<{t}xf16>
      %x = arith.extf %x16 : tensor<{t}xf16> to tensor<{t}xf32>
      %ninf = arith.constant 0xFF800000 : f32
      %m0 = tensor.splat %ninf : tensor<{chunk}xf32>
      %m = linalg.reduce {{ arith.maxnumf }} ins(%x : tensor<{t}xf32>) outs(%m0 : tensor<{chunk}xf32>) dimensions = [1]
      %e0 = tensor.empty() : tensor<{t}xf32>
      %e = linalg.generic {{indexing_maps = {bmaps}, iterator_types = ["parallel", "parallel"]}} ins(%x, %m : tensor<{t}xf32>, tensor<{chunk}xf32>) outs(%e0 : tensor<{t}xf32>) {{
      ^bb0(%a: f32, %b: f32, %o: f32):
        %d = arith.subf %a, %b : f32
        %v = math.exp %d : f32
        linalg.yield %v : f32
      }} -> tensor<{t}xf32>
      %zero = arith.constant 0.0 : f32
      %s0 = tensor.splat %zero : tensor<{chunk}xf32>
      %s = linalg.reduce {{ arith.addf }} ins(%e : tensor<{t}xf32>) outs(%s0 : tensor<{chunk}xf32>) dimensions = [1]
      %y0 = tensor.empty() : tensor<{t}xf32>
      %y = linalg.generic {{indexing_maps = {bmaps}, iterator_types = ["parallel", "parallel"]}} ins(%e, %s : tensor<{t}xf32>, tensor<{chunk}xf32>) outs(%y0 : tensor<{t}xf32>) {{
      ^bb0(%a: f32, %b: f32, %o: f32):
        %q = arith.divf %a, %b : f32
        linalg.yield %q : f32
      }} -> tensor<{t}xf32>
      %y16 = arith.truncf %y : tensor<{t}xf32> to tensor<{t}xf16>
      {_tile('%ot', '%ov', ['%r', '%c0'], (rows, cols), 'f16', (chunk, cols))}
      ktdp.store %y16, %ot : tensor<{t}xf16>, !ktdp.access_tile<{t}xindex>
      scf.yield
    }}
    return
  }}
}}
"""


def gemm(m: int = 4096, n: int = 4096, k: int = 4096, grid: Tuple[int, int] = (8, 4),
         bk: int = 128, sub: Tuple[int, int] = (128, 256)) -> str:
    gm, gn = grid
    assert m % gm == 0 and n % gn == 0 and k % bk == 0
    tm, tn = m // gm, n // gn
    sm, sn = min(sub[0], tm), min(sub[1], tn)
    assert tm % sm == 0 and tn % sn == 0
    at, bt, ct = f"{sm}x{bk}", f"{bk}x{sn}", f"{sm}x{sn}"
    return f"""module {{
  func.func @gemm_kernel(%a_ptr: index, %b_ptr: index, %c_ptr: index) attributes {{grid = [{gm}, {gn}]}} {{
    %pm, %pn = ktdp.get_compute_tile_id : index, index
    %c0 = arith.constant 0 : index
    %tm = arith.constant {tm} : index
    %tn = arith.constant {tn} : index
    %sm = arith.constant {sm} : index
    %sn = arith.constant {sn} : index
    %kk = arith.constant {k} : index
    %bk = arith.constant {bk} : index
    %m0 = arith.muli %pm, %tm : index
    %n0 = arith.muli %pn, %tn : index
    %m1 = arith.addi %m0, %tm : index
    %n1 = arith.addi %n0, %tn : index
{_view('%av', '%a_ptr', (m, k), 'f16')}{_view('%bv', '%b_ptr', (k, n), 'f16')}{_view('%cv', '%c_ptr', (m, n), 'f16')}
    scf.for %i = %m0 to %m1 step %sm {{
      scf.for %j = %n0 to %n1 step %sn {{
        %zero = arith.constant dense<0.0> : tensor<{ct}xf32>
        %acc = scf.for %kb = %c0 to %kk step %bk iter_args(%acc_in = %zero) -> (tensor<{ct}xf32>) {{
          {_tile('%at', '%av', ['%i', '%kb'], (m, k), 'f16', (sm, bk))}
          {_tile('%btile', '%bv', ['%kb', '%j'], (k, n), 'f16', (bk, sn))}
          %a16 = ktdp.load %at : !ktdp.access_tile<{at}xindex> -> tensor<{at}xf16>
          %b16 = ktdp.load %btile : !ktdp.access_tile<{bt}xindex> -> tensor<{bt}xf16>
          %a = arith.extf %a16 : tensor<{at}xf16> to tensor<{at}xf32>
          %b = arith.extf %b16 : tensor<{bt}xf16> to tensor<{bt}xf32>
          %acc_out = linalg.matmul ins(%a, %b : tensor<{at}xf32>, tensor<{bt}xf32>) outs(%acc_in : tensor<{ct}xf32>) -> tensor<{ct}xf32>
          scf.yield %acc_out : tensor<{ct}xf32>
        }}
        %c16 = arith.truncf %acc : tensor<{ct}xf32> to tensor<{ct}xf16>
        {_tile('%ct', '%cv', ['%i', '%j'], (m, n), 'f16', (sm, sn))}
        ktdp.store %c16, %ct : tensor<{ct}xf16>, !ktdp.access_tile<{ct}xindex>
        scf.yield
      }}
      scf.yield
    }}
    return
  }}
}}
"""


def gather_add(rows: int = 1048576, cols: int = 128, n_idx: int = 262144, grid: int = 64,
               chunk: int = 1024) -> str:
    assert n_idx % grid == 0
    per = n_idx // grid
    chunk = min(chunk, per)
    assert per % chunk == 0
    t = f"{chunk}x{cols}"
    return f"""module {{
  func.func @gather_add(%table_ptr: index, %idx_ptr: index) attributes {{grid = [{grid}]}} {{
    %core = ktdp.get_compute_tile_id : index
    %per = arith.constant {per} : index
    %step = arith.constant {chunk} : index
    %s0 = arith.muli %core, %per : index
    %s1 = arith.addi %s0, %per : index
{_view('%tv', '%table_ptr', (rows, cols), 'f16')}{_view('%xv', '%idx_ptr', (n_idx,), 'i32')}
    %one = arith.constant 1.0 : f16
    scf.for %s = %s0 to %s1 step %step {{
      %g = ktdp.construct_indirect_access_tile
          intermediate_variables(%gi, %gj)
          %tv[ind(%xv[%s + %gi]), (%gj)] {{
            variables_space_set = {_box((chunk, cols))},
            variables_space_order = {_ident(2)}
          }} : memref<{rows}x{cols}xf16>, memref<{n_idx}xi32> -> !ktdp.access_tile<{t}xindex>
      %rowsv = ktdp.load %g : !ktdp.access_tile<{t}xindex> -> tensor<{t}xf16>
      %upd = arith.addf %rowsv, %one : tensor<{t}xf16>
      ktdp.store %upd, %g : tensor<{t}xf16>, !ktdp.access_tile<{t}xindex>
      scf.yield
    }}
    return
  }}
}}
"""


def attention(batch: int = 4, heads: int = 32, seq: int = 2048, dim: int = 128, grid: int = 32,
              bq: int = 64, bk: int = 64, layout: str = "zigzag", groups: int = 1) -> str:
    """Causal attention; Q/K/V/O are [batch*heads*seq, dim] row-major views.

    layout "heads": core c owns heads [c*bh/grid, (c+1)*bh/grid), all query blocks.
    layout "zigzag": the query blocks of every head pair up as (b, nq-1-b), whose
    causal work sums to the same nq+1 key blocks; the pairs are dealt to the
    cores in order (with more cores than pairs, the heads of a pair are split
    between consecutive cores), so any contiguous range of cores owns the same
    amount of work and stretches of the sequence from both ends, and reads the
    K/V blocks of query blocks other cores own.
    groups > 1 (zigzag only): the heads form `groups` equal groups and the
    cores grid / groups equal rings; core c serves head group c // (grid /
    groups) and deals that group's zigzag pairs as above over the cores of
    its ring (part c % (grid / groups)), so the K/V blocks a core reads
    belong to cores of its own ring only."""
    bh = batch * heads
    assert seq % bq == 0 and bq == bk
    rows = bh * seq
    nq = seq // bq
    qt, kt, st = f"{bq}x{dim}", f"{bk}x{dim}", f"{bq}x{bk}"
    sc = 1.0 / float(np.sqrt(dim))
    rowmap = ("[affine_map<(d0, d1) -> (d0, d1)>, affine_map<(d0, d1) -> (d0)>, "
              "affine_map<(d0, d1) -> (d0, d1)>]")
    vecmap = ("[affine_map<(d0) -> (d0)>, affine_map<(d0) -> (d0)>, "
              "affine_map<(d0) -> (d0)>]")
    if layout == "heads":
        assert bh % grid == 0
        bounds = (f"    %per = arith.constant {bh // grid} : index\n"
                  "    %h0 = arith.muli %core, %per : index\n"
                  "    %h1 = arith.addi %h0, %per : index\n")
        loops = ("    scf.for %h = %h0 to %h1 step %c1 {\n"
                 "      %hbase = arith.muli %h, %seq : index\n"
                 "      scf.for %qb = %c0 to %nq step %c1 {\n")
        close = "        scf.yield\n      }\n      scf.yield\n    }\n"
    elif layout == "zigzag":
        assert nq % 2 == 0 and groups >= 1 and grid % groups == 0 and bh % groups == 0
        npairs = nq // 2
        parts, hg = grid // groups, bh // groups
        bounds = ""
        part = "%core"
        if groups > 1:
            # head group of the core's ring, and the core's place in that ring
            bounds = (f"    %parts = arith.constant {parts} : index\n"
                      f"    %hgroup = arith.constant {hg} : index\n"
                      "    %grp = arith.divsi %core, %parts : index\n"
                      "    %part = arith.remsi %core, %parts : index\n"
                      "    %gh0 = arith.muli %grp, %hgroup : index\n")
            part = "%part"
        if parts >= npairs:
            assert parts % npairs == 0 and hg % (parts // npairs) == 0
            split = parts // npairs
            bounds += (f"    %split = arith.constant {split} : index\n"
                       f"    %hper = arith.constant {hg // split} : index\n"
                       f"    %p0 = arith.divsi {part}, %split : index\n"
                       "    %p1 = arith.addi %p0, %c1 : index\n"
                       f"    %hpart = arith.remsi {part}, %split : index\n")
            if groups > 1:
                bounds += ("    %hrel = arith.muli %hpart, %hper : index\n"
                           "    %h0 = arith.addi %gh0, %hrel : index\n")
            else:
                bounds += "    %h0 = arith.muli %hpart, %hper : index\n"
            bounds += "    %h1 = arith.addi %h0, %hper : index\n"
        else:
            assert npairs % parts == 0
            bounds += (f"    %pper = arith.constant {npairs // parts} : index\n"
                       f"    %p0 = arith.muli {part}, %pper : index\n"
                       "    %p1 = arith.addi %p0, %pper : index\n")
            if groups > 1:
                bounds += ("    %h0 = arith.addi %gh0, %c0 : index\n"
                           "    %h1 = arith.addi %gh0, %hgroup : index\n")
            else:
                bounds += ("    %h0 = arith.constant 0 : index\n"
                           f"    %h1 = arith.constant {bh} : index\n")
        bounds += ("    %c2 = arith.constant 2 : index\n"
                   f"    %nqm1 = arith.constant {nq - 1} : index\n")
        loops = ("    scf.for %h = %h0 to %h1 step %c1 {\n"
                 "      %hbase = arith.muli %h, %seq : index\n"
                 "      scf.for %pp = %p0 to %p1 step %c1 {\n"
                 "        %pp2 = arith.muli %pp, %c2 : index\n"
                 "        %span = arith.subi %nqm1, %pp2 : index\n"
                 "        scf.for %side = %c0 to %c2 step %c1 {\n"
                 "        %jump = arith.muli %side, %span : index\n"
                 "        %qb = arith.addi %pp, %jump : index\n")
        close = ("        scf.yield\n      }\n        scf.yield\n      }\n"
                 "      scf.yield\n    }\n")
    else:
        raise ValueError(f"attention layout {layout!r}")
    if groups > 1 and layout != "zigzag":
        raise ValueError("head groups are a zigzag layout parameter")
    head = f"""module {{
  func.func @causal_attention(%q_ptr: index, %k_ptr: index, %v_ptr: index, %o_ptr: index) attributes {{grid = [{grid}]}} {{
    %core = ktdp.get_compute_tile_id : index
    %c0 = arith.constant 0 : index
    %c1 = arith.constant 1 : index
    %seq = arith.constant {seq} : index
    %nq = arith.constant {nq} : index
    %bq = arith.constant {bq} : index
    %scale = arith.constant {sc!r} : f32
    %ninf = arith.constant 0xFF800000 : f32
{_view('%qv', '%q_ptr', (rows, dim), 'f16')}{_view('%kv', '%k_ptr', (rows, dim), 'f16')}{_view('%vv', '%v_ptr', (rows, dim), 'f16')}{_view('%ov', '%o_ptr', (rows, dim), 'f16')}
"""
    body = f"""        %qoff = arith.muli %qb, %bq : index
        %qrow = arith.addi %hbase, %qoff : index
        {_tile('%qt', '%qv', ['%qrow', '%c0'], (rows, dim), 'f16', (bq, dim))}
        %q16 = ktdp.load %qt : !ktdp.access_tile<{qt}xindex> -> tensor<{qt}xf16>
        %q = arith.extf %q16 : tensor<{qt}xf16> to tensor<{qt}xf32>
        %m_init = tensor.splat %ninf : tensor<{bq}xf32>
        %fzero = arith.constant 0.0 : f32
        %l_init = tensor.splat %fzero : tensor<{bq}xf32>
        %acc_init = arith.constant dense<0.0> : tensor<{qt}xf32>
        %kend = arith.addi %qb, %c1 : index
        %m_fin, %l_fin, %acc_fin = scf.for %kb = %c0 to %kend step %c1
            iter_args(%m_i = %m_init, %l_i = %l_init, %acc_i = %acc_init)
            -> (tensor<{bq}xf32>, tensor<{bq}xf32>, tensor<{qt}xf32>) {{
          %koff = arith.muli %kb, %bq : index
          %krow = arith.addi %hbase, %koff : index
          {_tile('%ktile', '%kv', ['%krow', '%c0'], (rows, dim), 'f16', (bk, dim))}
          {_tile('%vtile', '%vv', ['%krow', '%c0'], (rows, dim), 'f16', (bk, dim))}
          %k16 = ktdp.load %ktile : !ktdp.access_tile<{kt}xindex> -> tensor<{kt}xf16>
          %v16 = ktdp.load %vtile : !ktdp.access_tile<{kt}xindex> -> tensor<{kt}xf16>
          %k = arith.extf %k16 : tensor<{kt}xf16> to tensor<{kt}xf32>
          %v = arith.extf %v16 : tensor<{kt}xf16> to tensor<{kt}xf32>
          %kT0 = tensor.empty() : tensor<{dim}x{bk}xf32>
          %kT = linalg.transpose ins(%k : tensor<{kt}xf32>) outs(%kT0 : tensor<{dim}x{bk}xf32>) permutation = [1, 0]
          %s0 = arith.constant dense<0.0> : tensor<{st}xf32>
          %sraw = linalg.matmul ins(%q, %kT : tensor<{qt}xf32>, tensor<{dim}x{bk}xf32>) outs(%s0 : tensor<{st}xf32>) -> tensor<{st}xf32>
          %ss = arith.mulf %sraw, %scale : tensor<{st}xf32>
          %sm0 = tensor.empty() : tensor<{st}xf32>
          %s = linalg.generic {{indexing_maps = [affine_map<(d0, d1) -> (d0, d1)>, affine_map<(d0, d1) -> (d0, d1)>], iterator_types = ["parallel", "parallel"]}} ins(%ss : tensor<{st}xf32>) outs(%sm0 : tensor<{st}xf32>) {{
          ^bb0(%x: f32, %o: f32):
            %ri = linalg.index 0 : index
            %ci = linalg.index 1 : index
            %rg = arith.addi %ri, %qoff : index
            %cg = arith.addi %ci, %koff : index
            %fut = arith.cmpi sgt, %cg, %rg : index
            %mx = arith.select %fut, %ninf, %x : f32
            linalg.yield %mx : f32
          }} -> tensor<{st}xf32>
          %mb0 = tensor.splat %ninf : tensor<{bq}xf32>
          %mb = linalg.reduce {{ arith.maxnumf }} ins(%s : tensor<{st}xf32>) outs(%mb0 : tensor<{bq}xf32>) dimensions = [1]
          %m_new = arith.maxnumf %m_i, %mb : tensor<{bq}xf32>
          %p0 = tensor.empty() : tensor<{st}xf32>
          %p = linalg.generic {{indexing_maps = {rowmap}, iterator_types = ["parallel", "parallel"]}} ins(%s, %m_new : tensor<{st}xf32>, tensor<{bq}xf32>) outs(%p0 : tensor<{st}xf32>) {{
          ^bb0(%x: f32, %mm: f32, %o: f32):
            %dx = arith.subf %x, %mm : f32
            %ex = math.exp %dx : f32
            linalg.yield %ex : f32
          }} -> tensor<{st}xf32>
          %al0 = tensor.empty() : tensor<{bq}xf32>
          %alpha = linalg.generic {{indexing_maps = {vecmap}, iterator_types = ["parallel"]}} ins(%m_i, %m_new : tensor<{bq}xf32>, tensor<{bq}xf32>) outs(%al0 : tensor<{bq}xf32>) {{
          ^bb0(%mo: f32, %mn: f32, %o: f32):
            %dm = arith.subf %mo, %mn : f32
            %em = math.exp %dm : f32
            linalg.yield %em : f32
          }} -> tensor<{bq}xf32>
          %ps0 = tensor.splat %fzero : tensor<{bq}xf32>
          %psum = linalg.reduce {{ arith.addf }} ins(%p : tensor<{st}xf32>) outs(%ps0 : tensor<{bq}xf32>) dimensions = [1]
          %l_sc = arith.mulf %l_i, %alpha : tensor<{bq}xf32>
          %l_new = arith.addf %l_sc, %psum : tensor<{bq}xf32>
          %ac0 = tensor.empty() : tensor<{qt}xf32>
          %acc_sc = linalg.generic {{indexing_maps = {rowmap}, iterator_types = ["parallel", "parallel"]}} ins(%acc_i, %alpha : tensor<{qt}xf32>, tensor<{bq}xf32>) outs(%ac0 : tensor<{qt}xf32>) {{
          ^bb0(%x: f32, %al: f32, %o: f32):
            %xs = arith.mulf %x, %al : f32
            linalg.yield %xs : f32
          }} -> tensor<{qt}xf32>
          %acc_new = linalg.matmul ins(%p, %v : tensor<{st}xf32>, tensor<{kt}xf32>) outs(%acc_sc : tensor<{qt}xf32>) -> tensor<{qt}xf32>
          scf.yield %m_new, %l_new, %acc_new : tensor<{bq}xf32>, tensor<{bq}xf32>, tensor<{qt}xf32>
        }}
        %on0 = tensor.empty() : tensor<{qt}xf32>
        %on = linalg.generic {{indexing_maps = {rowmap}, iterator_types = ["parallel", "parallel"]}} ins(%acc_fin, %l_fin : tensor<{qt}xf32>, tensor<{bq}xf32>) outs(%on0 : tensor<{qt}xf32>) {{
        ^bb0(%x: f32, %ll: f32, %o: f32):
          %xo = arith.divf %x, %ll : f32
          linalg.yield %xo : f32
        }} -> tensor<{qt}xf32>
        %o16 = arith.truncf %on : tensor<{qt}xf32> to tensor<{qt}xf16>
        {_tile('%otile', '%ov', ['%qrow', '%c0'], (rows, dim), 'f16', (bq, dim))}
        ktdp.store %o16, %otile : tensor<{qt}xf16>, !ktdp.access_tile<{qt}xindex>
"""
    return head + bounds + loops + body + close + "    return\n  }\n}\n"


# ---------------------------------------------------------------------------
# seeded inputs (shapes and distributions of the benchmark configurations)
# ---------------------------------------------------------------------------

FULL = {
    "vector_add": dict(n=1024, grid=1),
    "softmax": dict(rows=4096, cols=1024, grid=32, chunk=32),
    "gemm": dict(m=4096, n=4096, k=4096, grid=(8, 4)),
    "gather_add": dict(rows=1048576, cols=128, n_idx=262144, grid=64, chunk=1024),
    # 32 cores: 4 head groups (32 of the 128 heads each), each served by a ring
    # of 8 cores that own zigzag query-block pairs and read each other's K/V
    "attention": dict(batch=4, heads=32, seq=2048, dim=128, grid=32, groups=4),
}

FUNC = {"vector_add": "add_kernel", "softmax": "softmax_rows", "gemm": "gemm_kernel",
        "gather_add": "gather_add", "attention": "causal_attention"}

SOURCE = {"vector_add": vector_add, "softmax": softmax, "gemm": gemm,
          "gather_add": gather_add, "attention": attention}


def inputs(name: str, seed: int = 0, **p) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    cfg = dict(FULL[name])
    cfg.update(p)
    if name == "vector_add":
        n = cfg["n"]
        return {"x_ptr": rng.standard_normal(n).astype(np.float16),
                "y_ptr": rng.standard_normal(n).astype(np.float16),
                "out_ptr": np.zeros(n, np.float16)}
    if name == "softmax":
        shape = (cfg["rows"], cfg["cols"])
        return {"in_ptr": (2 * rng.standard_normal(shape)).astype(np.float16),
                "out_ptr": np.zeros(shape, np.float16)}
    if name == "gemm":
        m, n, k = cfg["m"], cfg["n"], cfg["k"]
        return {"a_ptr": rng.uniform(-1, 1, (m, k)).astype(np.float16),
                "b_ptr": rng.uniform(-1, 1, (k, n)).astype(np.float16),
                "c_ptr": np.zeros((m, n), np.float16)}
    if name == "gather_add":
        return {"table_ptr": rng.standard_normal((cfg["rows"], cfg["cols"])).astype(np.float16),
                "idx_ptr": rng.integers(0, cfg["rows"], cfg["n_idx"]).astype(np.int32)}
    if name == "attention":
        rows = cfg["batch"] * cfg["heads"] * cfg["seq"]
        d = cfg["dim"]
        return {"q_ptr": rng.standard_normal((rows, d)).astype(np.float16),
                "k_ptr": rng.standard_normal((rows, d)).astype(np.float16),
                "v_ptr": rng.standard_normal((rows, d)).astype(np.float16),
                "o_ptr": np.zeros((rows, d), np.float16)}
    raise KeyError(name)


def source(name: str, **p) -> str:
    cfg = dict(FULL[name])
    cfg.update(p)
    return SOURCE[name](**cfg)
