"""Writes the structure-input fixtures under tests/golden/structures/.

They are synthetic: backbones from the seeded ideal-geometry generator
(hkb_synthetic_backbone), written as PDB / mmCIF text with the cases the
reference's normaliser distinguishes (io/structure_normalize.cpp):
altlocs, insertion codes, numbering gaps, several models and chains, waters
and ligands, a modified residue read as its parent (MSE), glycines with and
without CB, side-chain / OXT atoms to strip, residues missing atoms (some
inferable by the rigid template fit, some not), and, for mmCIF, quoted
tokens and a row wrapped over two lines.  The tests load each file with this
package's loader and with the reference's own (oracle/_ref) and require
identical output.

Run from the repository root:  python tests/golden/make_structures.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent / "structures"

THREE = ["ALA", "ARG", "ASN", "ASP", "CYS", "GLN", "GLU", "GLY", "HIS", "ILE",
         "LEU", "LYS", "MET", "PHE", "PRO", "SER", "THR", "TRP", "TYR", "VAL"]
NAMES = ["N", "CA", "C", "O", "CB"]


def backbone(seed: int, L: int):
    from hikoboshi_b200 import synthetic_backbone
    c, _ = synthetic_backbone(seed, L)
    return c


def pdb_atom(serial, name, resname, chain, resnum, x, y, z, het=False, alt=" ", icode=" ",
             elem=None):
    rec = "HETATM" if het else "ATOM  "
    nm = (" " + name).ljust(4) if len(name) < 4 else name
    elem = elem or name[0]
    return (f"{rec}{serial:5d} {nm}{alt}{resname:>3s} {chain}{resnum:4d}{icode}   "
            f"{x:8.3f}{y:8.3f}{z:8.3f}{1.00:6.2f}{20.00:6.2f}          {elem:>2s}")


def residue_atoms(coords, i, resname, drop=()):
    """(name, xyz) of residue i: backbone (CB omitted for GLY) + a side-chain atom."""
    out = []
    for k, nm in enumerate(NAMES):
        if nm in drop or (nm == "CB" and resname == "GLY"):
            continue
        out.append((nm, coords[i, k]))
    if resname not in ("GLY", "ALA"):
        out.append(("CG", coords[i, 4] + np.array([0.9, 0.7, -0.8], np.float32)))
    return out


def write_basic(path: Path):
    c = backbone(5, 60)
    lines, serial = [], 1
    for i in range(60):
        rn = THREE[i % 20]
        for nm, xyz in residue_atoms(c, i, rn):
            lines.append(pdb_atom(serial, nm, rn, "A", i + 1, *xyz))
            serial += 1
    lines.append(pdb_atom(serial, "OXT", THREE[59 % 20], "A", 60, *(c[59, 3] + 1.1), elem="O"))
    lines += ["TER", "END"]
    path.write_text("\n".join(lines) + "\n")


def template_residue(at: np.ndarray) -> np.ndarray:
    """The reference loader's ideal residue (io/residue_table.cpp:61-115: N on
    -x, C at angle 1.9416 - pi/2 in the xy plane, O, CB by the virtual-CB rule),
    rotated and moved to `at`: a residue whose rigid template fit passes the
    0.5 A guard, so a dropped atom is inferred."""
    f = np.float32
    n = np.array([-1.458, 0, 0], f)
    ca = np.zeros(3, f)
    c = np.array([1.525 * np.cos(1.9416 - np.pi / 2), 1.525 * np.sin(1.9416 - np.pi / 2), 0], f)
    u = c / np.linalg.norm(c)
    w = np.array([-u[1], u[0], 0], f)
    d = np.cos(np.pi - 2.1031) * u + np.sin(np.pi - 2.1031) * w
    o = c + 1.231 * d
    b, cv = ca - n, c - ca
    cb = ca - 0.58273431 * np.cross(b, cv) + 0.56802827 * b - 0.54067466 * cv
    th = 0.7
    rot = np.array([[np.cos(th), -np.sin(th), 0], [np.sin(th), np.cos(th), 0], [0, 0, 1]], f)
    return (np.stack([n, ca, c, o, cb]) @ rot.T + at).astype(np.float32)


def write_messy(path: Path):
    c1 = backbone(9, 40)
    c1[8] = template_residue(c1[8, 1])
    c2 = backbone(10, 30)
    lines, serial = ["HEADER    SYNTHETIC TEST STRUCTURE"], 1
    for model, shift in ((1, 0.0), (2, 0.25)):
        lines.append(f"MODEL     {model:4d}")
        # chain B first in file order, then chain A: the default picks A
        for i in range(30):
            rn = THREE[(3 * i) % 20]
            for nm, xyz in residue_atoms(c2, i, rn):
                lines.append(pdb_atom(serial, nm, rn, "B", i + 1, *(xyz + shift)))
                serial += 1
        num = 0
        for i in range(40):
            rn = THREE[(7 * i + 1) % 20]
            num += 1
            icode = " "
            if i == 12:
                num += 5                      # numbering gap
            if i == 20:
                num -= 1
                icode = "A"                   # insertion code: 21A after 21
            drop = ()
            if i == 8:
                drop = ("O",)                 # inferable: the residue is the template
            if i == 15:
                drop = ("N", "CA", "C")       # too few anchors: stays missing
            if i == 25:
                rn = "GLY"
                drop = ("N",)                 # glycine CB from partial anchors
            het = i == 30
            if het:
                rn = "MSE"
            for nm, xyz in residue_atoms(c1, i, rn, drop):
                xyz = xyz + shift
                if i in (5, 6) and nm in ("CA", "C"):
                    # altlocs: B first then A (A must win), and a blank after A
                    lines.append(pdb_atom(serial, nm, rn, "A", num, *(xyz + 0.3), het, "B", icode))
                    serial += 1
                    lines.append(pdb_atom(serial, nm, rn, "A", num, *xyz, het, "A", icode))
                    serial += 1
                    if i == 6:
                        lines.append(pdb_atom(serial, nm, rn, "A", num, *(xyz - 0.2), het, " ",
                                              icode))
                        serial += 1
                    continue
                lines.append(pdb_atom(serial, nm, rn, "A", num, *xyz, het, " ", icode))
                serial += 1
        for w in range(3):
            lines.append(pdb_atom(serial, "O", "HOH", "A", 500 + w, 10.0 + w, 5.0, -3.0, True,
                                  elem="O"))
            serial += 1
        lines.append(pdb_atom(serial, "C1", "LIG", "C", 900, 1.0, 2.0, 3.0, True, elem="C"))
        serial += 1
        lines.append("ENDMDL")
    lines.append("END")
    path.write_text("\n".join(lines) + "\n")


def write_no_chain_a(path: Path):
    c = backbone(12, 25)
    lines, serial = [], 1
    for chain, lo, hi in (("D", 0, 12), ("E", 12, 25)):
        for i in range(lo, hi):
            rn = THREE[(i * 11) % 20]
            for nm, xyz in residue_atoms(c, i, rn):
                lines.append(pdb_atom(serial, nm, rn, chain, i + 1, *xyz))
                serial += 1
    path.write_text("\n".join(lines) + "\n")


def write_cif(path: Path):
    c = backbone(21, 35)
    cols = ["group_PDB", "id", "type_symbol", "label_atom_id", "label_alt_id", "label_comp_id",
            "label_asym_id", "label_seq_id", "pdbx_PDB_ins_code", "Cartn_x", "Cartn_y",
            "Cartn_z", "occupancy", "auth_seq_id", "auth_comp_id", "auth_asym_id",
            "auth_atom_id", "pdbx_PDB_model_num"]
    lines = ["data_SYNTH", "#", "_entry.id SYNTH", "#", "loop_"]
    lines += [f"_atom_site.{n}" for n in cols]
    serial = 1
    for i in range(35):
        rn = THREE[(5 * i + 2) % 20]
        drop = ("O", "CB") if i == 9 else ()
        for nm, xyz in residue_atoms(c, i, rn, drop):
            alt = "."
            row = ["ATOM", str(serial), nm[0], f'"{nm}"' if nm == "CA" else nm, alt, rn, "A",
                   str(i + 1), "?", f"{xyz[0]:.3f}", f"{xyz[1]:.3f}", f"{xyz[2]:.3f}", "1.00",
                   str(i + 101), rn, "A", nm, "1"]
            if serial == 7:
                lines.append(" ".join(row[:9]))    # a row wrapped over two lines
                lines.append(" ".join(row[9:]))
            else:
                lines.append(" ".join(row))
            serial += 1
    lines += ["#", "loop_", "_struct_conf.id", "HELX1", "#"]
    path.write_text("\n".join(lines) + "\n")


def main():
    OUT.mkdir(exist_ok=True)
    write_basic(OUT / "basic_L60.pdb")
    write_messy(OUT / "models_chains_altlocs.pdb")
    write_no_chain_a(OUT / "chains_D_E.pdb")
    write_cif(OUT / "synth_L35.cif")
    (OUT / "bad_coordinate.pdb").write_text(
        "ATOM      1  N   ALA A   1      11.104  x6.134  -6.504  1.00  0.00           N\n")
    (OUT / "short_record.pdb").write_text("ATOM      1  N   ALA A   1      11.104\n")
    (OUT / "waters_only.pdb").write_text(
        pdb_atom(1, "O", "HOH", "A", 1, 1.0, 2.0, 3.0, True, elem="O") + "\n")
    (OUT / "no_atoms.txt").write_text("just some text\n")
    print("wrote", sorted(p.name for p in OUT.iterdir()))


if __name__ == "__main__":
    main()
