"""Detection comparison at the reference's DetectorOptions defaults (confidence
0.25, IoU 0.45, Vision/YoloDecoder.cs:25-28) between a device output and the
oracle's, for one image's [4 + nc, anchors] head output.

Detections. A random-init detector's class scores sit in a narrow band (about
0.506-0.514 here), so thousands of candidates differ by less than 1e-6 and
their sort order is decided by rounding. The comparison therefore checks each
decision the reference makes and flags (reports, does not hide) the ones that
lie within the parity tolerance of a threshold or of a tie:
  1. candidates: the same anchors pass `best >= conf` with the same class,
     except anchors whose score is within 1e-4 of conf or whose top two class
     scores are within 1e-6 (flagged);
  2. order: every pair the two outputs sort differently has scores within 1e-6
     of each other (flagged as ties);
  3. suppression: walking the reference's candidates in the reference's order
     against the reference's kept boxes, the GPU boxes make the same
     keep/suppress decision, except where the deciding IoU is within 1e-4 of
     the threshold (flagged);
  4. the two independent NMS runs are reported identical or not; they must be
     identical whenever nothing was flagged in 1-3."""
from __future__ import annotations

import numpy as np

CONF, IOU = 0.25, 0.45          # DetectorOptions defaults (YoloDecoder.cs:25-28)
NEAR = 1e-4                      # "within 1e-4 of a threshold" is flagged
TIE = 1e-6                       # score differences at or below this are ties (measured error ~1e-7)
F = np.float32


def _candidates(out):
    scores = out[4:]
    cls = np.argmax(scores, axis=0)
    best = scores[cls, np.arange(out.shape[1])]
    top2 = np.partition(scores, -2, axis=0)[-2]
    ok = np.isfinite(best) & (best >= F(CONF)) & np.all(np.isfinite(out[:4]), axis=0) & (out[2] > 0) & (out[3] > 0)
    return cls, best, best - top2, ok


def _xywh(out, idx):
    x, y, w, h = (out[i, idx].astype(F) for i in range(4))
    return np.stack([(x - w * F(0.5)).astype(F), (y - h * F(0.5)).astype(F), w, h], 1)


def _iou(box, kept):
    """Detection.IoU (Detection.cs:31-50) of one box against many, float32 op by op."""
    x1 = np.maximum(box[0], kept[:, 0])
    y1 = np.maximum(box[1], kept[:, 1])
    x2 = np.minimum((box[0] + box[2]).astype(F), (kept[:, 0] + kept[:, 2]).astype(F))
    y2 = np.minimum((box[1] + box[3]).astype(F), (kept[:, 1] + kept[:, 3]).astype(F))
    iw, ih = (x2 - x1).astype(F), (y2 - y1).astype(F)
    inter = (iw * ih).astype(F)
    union = ((F(box[2] * box[3]) + (kept[:, 2] * kept[:, 3]).astype(F)).astype(F) - inter).astype(F)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = np.where((iw > 0) & (ih > 0) & (union > 0), (inter / union).astype(F), F(0))
    return v


def _nms(order, cls, boxes, max_det=300, forced=None):
    """Greedy per-class NMS over candidates in `order`; returns kept anchors and
    each visited candidate's deciding IoU (max IoU against the kept boxes of its
    class). With `forced` (anchor -> kept?) the kept set follows those decisions."""
    kept, kept_boxes, kept_cls, decide = [], [], [], {}
    for a in order:
        if kept_boxes:
            kb = np.asarray(kept_boxes, F)
            same = np.asarray(kept_cls) == cls[a]
            m = float(_iou(boxes[a], kb[same]).max()) if same.any() else 0.0
        else:
            m = 0.0
        decide[a] = m
        keep = (m <= IOU) if forced is None else forced[a]
        if keep:
            kept.append(a)
            kept_boxes.append(boxes[a])
            kept_cls.append(cls[a])
            if len(kept) >= max_det:
                break
    return kept, decide


def compare_detections(out, ref):
    """Returns (report dict, list of unflagged disagreements)."""
    rc, rb, rgap, rok = _candidates(ref)
    gc, gb, ggap, gok = _candidates(out)
    A = ref.shape[1]
    bad = []
    near_conf = (np.abs(rb - F(CONF)) <= NEAR) | (np.abs(gb - F(CONF)) <= NEAR)
    cls_tie = (rgap <= TIE) | (ggap <= TIE)
    diff_cand = np.nonzero(rok != gok)[0]
    diff_cls = np.nonzero(rok & gok & (rc != gc))[0]
    bad += [("candidate", int(a)) for a in diff_cand if not near_conf[a]]
    bad += [("class", int(a)) for a in diff_cls if not cls_tie[a]]
    cand = np.nonzero(rok & gok)[0]
    r_order = cand[np.lexsort((cand, -rb[cand]))]
    g_order = cand[np.lexsort((cand, -gb[cand]))]
    # 2. order: positions where the sorted lists differ must be ties in score
    inv = np.nonzero(r_order != g_order)[0]
    order_ties = 0
    for i in inv:
        a, b = r_order[i], g_order[i]
        if abs(float(rb[a]) - float(rb[b])) <= TIE and abs(float(gb[a]) - float(gb[b])) <= TIE:
            order_ties += 1
        else:
            bad.append(("order", int(a), int(b)))
    # 3. suppression decisions along the reference's path
    r_boxes = np.zeros((A, 4), F)
    g_boxes = np.zeros((A, 4), F)
    r_boxes[cand] = _xywh(ref, cand)
    g_boxes[cand] = _xywh(out, cand)
    r_kept, r_dec = _nms(r_order, rc, r_boxes)
    forced = {a: (r_dec[a] <= IOU) for a in r_dec}
    _, g_dec = _nms(r_order, rc, g_boxes, forced=forced)
    near_iou = 0
    for a, m in r_dec.items():
        gm = g_dec.get(a, m)
        if (m <= IOU) != (gm <= IOU):
            if abs(m - IOU) <= NEAR or abs(gm - IOU) <= NEAR:
                near_iou += 1
            else:
                bad.append(("suppression", int(a), m, gm))
        elif abs(m - IOU) <= NEAR:
            near_iou += 1
    # 4. independent runs
    g_kept, _ = _nms(g_order, gc, g_boxes)
    identical = r_kept == g_kept and np.allclose(r_boxes[r_kept], g_boxes[g_kept], rtol=1e-4, atol=1e-3)
    flagged = int(near_conf[rok | gok].sum()) + int(cls_tie[rok | gok].sum()) + order_ties + near_iou
    if not identical and flagged == 0:
        bad.append(("lists differ with nothing flagged",))
    rep = dict(candidates=int(len(cand)), kept=len(r_kept), identical=bool(identical), near_conf=int(
        near_conf[rok | gok].sum()), class_ties=int(cls_tie[rok | gok].sum()), order_ties=order_ties,
        near_iou=near_iou)
    return rep, bad
